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

// Codes are stored G-major: value 256 b + 32 G + 8 o + j (block b, group
// G of 32, octet o, byte j) sits at byte G * (n/8) + 8 * (4 b + o) + j of
// hi / lo, and the octet sums of (b, G, o) at G * (n/64) + 4 b + o.  A
// reader lane owns (b, o) (lane = 4 b + o within its row group) and loads
// all eight G, so for each G the lanes of a warp read one contiguous run:
// no shared-memory bank conflicts (block-major order put the 8 blocks 256
// bytes apart, 8 lanes on one bank, while every warp of the CTA loads its
// codes at the same time).
struct QVec {
    int8_t* hi;
    int8_t* lo;
    float* s;     // [n/256] block scales
    int16_t* oh;  // [n/8] octet sums of hi
    int16_t* ol;  // [n/8] octet sums of lo
    int n8;       // n / 8: bytes of one G plane of hi / lo
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
    q.n8 = n / 8;
    return q;
}

// Quantise one 256-value block b with one warp, lane l holding values
// 8l..8l+7 (octet l) in `vals`.  No block-wide barrier; the caller
// synchronises before the codes are read.
__device__ __forceinline__ void quantize_block_vals(const float (&vals)[8], QVec q, int b) {
    const int lane = threadIdx.x & 31;
    float m = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) m = fmaxf(m, fabsf(vals[e]));
    // the magnitudes are non-negative, so their bit patterns order like the
    // values: one redux.sync instead of five shuffle rounds
    m = __uint_as_float(__reduce_max_sync(0xffffffffu, __float_as_uint(m)));
    float iv;
    if (!(m <= 3.0e38f)) {  // inf / nan in the block: propagate as nan
        iv = 0.f;
        if (lane == 0) q.s[b] = __int_as_float(0x7fc00000);
    } else {
        // fast division: a code may be off by one unit; the scale stored
        // with the codes is what the dot products use
        iv = m > 0.f ? (m < 1e37f ? __fdividef(32512.f, m) : 32512.f / m) : 0.f;
        if (lane == 0) q.s[b] = m * (1.0f / 32512.f);
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
    const int G = lane >> 2, o = lane & 3;
    const int off = G * q.n8 + 8 * (4 * b + o), oc = G * (q.n8 >> 3) + 4 * b + o;
    *reinterpret_cast<uint2*>(q.hi + off) = make_uint2(ph[0], ph[1]);
    *reinterpret_cast<uint2*>(q.lo + off) = make_uint2(pl[0], pl[1]);
    q.oh[oc] = (int16_t)sh;
    q.ol[oc] = (int16_t)sl;
}

// Block b of an fp32 vector in shared memory.
__device__ __forceinline__ void quantize_block_warp(const float* v, QVec q, int b) {
    const int lane = threadIdx.x & 31;
    const float4 a0 = *reinterpret_cast<const float4*>(v + 256 * b + 8 * lane);
    const float4 a1 = *reinterpret_cast<const float4*>(v + 256 * b + 8 * lane + 4);
    const float vals[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    quantize_block_vals(vals, q, b);
}

// The same, out of line (one copy per kernel that needs a small step).
static __device__ __noinline__ void quantize_block_ool(const float* v, uint8_t* codes, int n, int b) {
    quantize_block_warp(v, qvec_at(codes, n), b);
}

// Block b of an fp32 vector in global memory written by other CTAs of this
// launch (read through L2).
__device__ __forceinline__ void quantize_block_gmem(const float* v, QVec q, int b) {
    const int lane = threadIdx.x & 31;
    const float4 a0 = __ldcg(reinterpret_cast<const float4*>(v + 256 * b + 8 * lane));
    const float4 a1 = __ldcg(reinterpret_cast<const float4*>(v + 256 * b + 8 * lane + 4));
    const float vals[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    quantize_block_vals(vals, q, b);
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
        const int off = G * v.n8 + 8 * (4 * b + o), oc = G * (v.n8 >> 3) + 4 * b + o;
        const uint2 hh = *reinterpret_cast<const uint2*>(v.hi + off);
        const uint2 ll = *reinterpret_cast<const uint2*>(v.lo + off);
        x.h[G][0] = hh.x;
        x.h[G][1] = hh.y;
        x.l[G][0] = ll.x;
        x.l[G][1] = ll.y;
        x.sh8[G] = v.oh[oc];
        x.sl8[G] = v.ol[oc];
    }
    x.s = v.s[b];
}

__device__ __forceinline__ int dp4(uint32_t a, uint32_t b, int c) {
    return __dp4a((int)a, (int)b, c);
}

// ---- per-format partial dot of one lane's 64 values (block pointer bp) ----
//
// Shared-memory loads are the scarce resource here (one warp-wide load issue
// per SM cycle), so every decoder reads its bytes with the widest aligned
// loads the block layout allows and extracts fields in registers.  Blocks of
// 110 (Q3_K) and 210 (Q6_K) bytes are only 2-byte aligned: their words are
// read as aligned words and funnel-shifted by 0 or 16 bits.

__device__ __forceinline__ uint32_t lds32(const uint8_t* p) {
    return *reinterpret_cast<const uint32_t*>(p);
}

// Two consecutive 32-bit words starting at a 2-byte aligned address:
// al = address rounded down to 4, sh = 8 * (address & 3) in {0, 16}.
__device__ __forceinline__ uint2 lds64_a2(const uint8_t* al, int sh) {
    const uint32_t w0 = lds32(al), w1 = lds32(al + 4), w2 = lds32(al + 8);
    return make_uint2(__funnelshift_r(w0, w1, sh), __funnelshift_r(w1, w2, sh));
}

__device__ __forceinline__ float h2f(uint32_t bits16) {
    return __half2float(__ushort_as_half((unsigned short)(bits16 & 0xFFFFu)));
}


// Zero-extended byte i of w (one PRMT).
__device__ __forceinline__ int ubyte(uint32_t w, int i) { return (int)__byte_perm(w, 0u, 0x4440u | (uint32_t)i); }
// Sign-extended byte i of w: one PRMT whose selector nibbles 1..3 have
// their msb set, which replicates the sign bit of byte i (PTX prmt, generic
// mode).
__device__ __forceinline__ int sbyte(uint32_t w, int i) {
    const uint32_t sel = (uint32_t)i | ((uint32_t)(8 | i) << 4) | ((uint32_t)(8 | i) << 8) |
                         ((uint32_t)(8 | i) << 12);
    uint32_t r;
    asm("prmt.b32 %0, %1, 0, %2;" : "=r"(r) : "r"(w), "r"(sel));
    return (int)r;
}

// Q3_K: u = q + 4 in 0..7; 13 shared loads per lane.  The -4 * sum(x)
// correction rides in the dp4a accumulator's start value.
__device__ __forceinline__ float qdot_q3k(const uint8_t* bp, int o, const XLane& x) {
    const uint8_t* al = reinterpret_cast<const uint8_t*>((uintptr_t)bp & ~(uintptr_t)3);
    const int sh = 8 * (int)((uintptr_t)bp & 3);
    const uint2 hm = lds64_a2(al + 8 * o, sh);
    const uint2 qa = lds64_a2(al + 32 + 8 * o, sh);
    const uint2 qb = lds64_a2(al + 64 + 8 * o, sh);
    const uint32_t w0 = lds32(al + 96), w1 = lds32(al + 100), w2 = lds32(al + 104), w3 = lds32(al + 108);
    const uint32_t s03 = __funnelshift_r(w0, w1, sh), s47 = __funnelshift_r(w1, w2, sh);
    const uint32_t s811 = __funnelshift_r(w2, w3, sh);
    const float d = h2f(w3 >> sh);
    // six-bit scales j = 2G + jo (reference dequant_q3_k, cpp/dequant_k.cpp:284-289),
    // as signed bytes (scale - 32)
    const int jo = o >> 1;
    const uint32_t bq = __byte_perm(s03, s47, jo | ((2 + jo) << 4) | ((4 + jo) << 8) | ((6 + jo) << 12));
    const uint32_t t = __byte_perm(s811, 0u, jo | ((2 + jo) << 4) | (jo << 8) | ((2 + jo) << 12));
    const uint32_t hiA = (t & 0x00000303u) | ((t >> 2) & 0x03030000u);
    const uint32_t hiB = ((t >> 4) & 0x00000303u) | ((t >> 6) & 0x03030000u);
    uint32_t scA = ((bq & 0x0F0F0F0Fu) | (hiA << 4)) ^ 0x20202020u;          // 6-bit two's complement
    uint32_t scB = (((bq >> 4) & 0x0F0F0F0Fu) | (hiB << 4)) ^ 0x20202020u;
    scA |= (scA & 0x20202020u) * 6u;                                          // sign-extend to 8 bits
    scB |= (scB & 0x20202020u) * 6u;
    int ah = 0, alo = 0;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint32_t q0 = G < 4 ? qa.x : qb.x, q1 = G < 4 ? qa.y : qb.y;
        const int s2 = 2 * (G & 3);
        // hmask bit G of each byte moved to bit 2 (one shift, one mask)
        const uint32_t hb0 = (G >= 2 ? hm.x >> (G - 2) : hm.x << (2 - G)) & 0x04040404u;
        const uint32_t hb1 = (G >= 2 ? hm.y >> (G - 2) : hm.y << (2 - G)) & 0x04040404u;
        const uint32_t u0 = ((q0 >> s2) & 0x03030303u) | hb0;
        const uint32_t u1 = ((q1 >> s2) & 0x03030303u) | hb1;
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(u1, xh.y, dp4(u0, xh.x, -4 * x.sh(G)));
        const int l = dp4(u1, xl.y, dp4(u0, xl.x, -4 * x.sl(G)));
        const int sc = sbyte(G < 4 ? scA : scB, G & 3);
        ah += sc * h;
        alo += sc * l;
    }
    return d * x.s * fmaf(256.f, (float)ah, (float)alo);
}

// (scale, min) bytes of Q4_K/Q5_K sub-blocks 0..3 and 4..7 from the 12
// packed bytes (reference unpack_scale_min_k4, cpp/dequant_k.cpp:166-175):
// y = bytes 0..3, z = bytes 4..7, w = bytes 8..11.
__device__ __forceinline__ void k4_scales_words(uint32_t y, uint32_t z, uint32_t w, uint32_t& sc03,
                                                uint32_t& mn03, uint32_t& sc47, uint32_t& mn47) {
    sc03 = y & 0x3F3F3F3Fu;
    mn03 = z & 0x3F3F3F3Fu;
    sc47 = (w & 0x0F0F0F0Fu) | ((y >> 2) & 0x30303030u);
    mn47 = ((w >> 4) & 0x0F0F0F0Fu) | ((z >> 2) & 0x30303030u);
}

// Q4_K: 16-byte aligned blocks; 5 shared loads per lane.
__device__ __forceinline__ float qdot_q4k(const uint8_t* bp, int o, const XLane& x) {
    const uint4 hd = *reinterpret_cast<const uint4*>(bp);
    uint32_t sc03, mn03, sc47, mn47;
    k4_scales_words(hd.y, hd.z, hd.w, sc03, mn03, sc47, mn47);
    int ah = 0, alo = 0, mh = 0, ml = 0;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
        const uint2 w = *reinterpret_cast<const uint2*>(bp + 16 + 32 * pp + 8 * o);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int G = 2 * pp + hf;
            const uint32_t u0 = (w.x >> (4 * hf)) & 0x0F0F0F0Fu, u1 = (w.y >> (4 * hf)) & 0x0F0F0F0Fu;
            const uint2 xh = x.h2(G), xl = x.l2(G);
            const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
            const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
            const int sc = ubyte(G < 4 ? sc03 : sc47, G & 3);
            const int mn = ubyte(G < 4 ? mn03 : mn47, G & 3);
            ah += sc * h;
            alo += sc * l;
            mh += mn * x.sh(G);
            ml += mn * x.sl(G);
        }
    }
    const float a = fmaf(256.f, (float)ah, (float)alo);
    const float m = fmaf(256.f, (float)mh, (float)ml);
    return x.s * (h2f(hd.x) * a - h2f(hd.x >> 16) * m);
}

// Q5_K: 16-byte aligned blocks; 6 shared loads per lane.
__device__ __forceinline__ float qdot_q5k(const uint8_t* bp, int o, const XLane& x) {
    const uint4 hd = *reinterpret_cast<const uint4*>(bp);
    uint32_t sc03, mn03, sc47, mn47;
    k4_scales_words(hd.y, hd.z, hd.w, sc03, mn03, sc47, mn47);
    const uint2 qh = *reinterpret_cast<const uint2*>(bp + 16 + 8 * o);
    int ah = 0, alo = 0, mh = 0, ml = 0;
#pragma unroll
    for (int pp = 0; pp < 4; ++pp) {
        const uint2 w = *reinterpret_cast<const uint2*>(bp + 48 + 32 * pp + 8 * o);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int G = 2 * pp + hf;
            const uint32_t u0 = ((w.x >> (4 * hf)) & 0x0F0F0F0Fu) | (((qh.x >> G) & 0x01010101u) << 4);
            const uint32_t u1 = ((w.y >> (4 * hf)) & 0x0F0F0F0Fu) | (((qh.y >> G) & 0x01010101u) << 4);
            const uint2 xh = x.h2(G), xl = x.l2(G);
            const int h = dp4(u1, xh.y, dp4(u0, xh.x, 0));
            const int l = dp4(u1, xl.y, dp4(u0, xl.x, 0));
            const int sc = ubyte(G < 4 ? sc03 : sc47, G & 3);
            const int mn = ubyte(G < 4 ? mn03 : mn47, G & 3);
            ah += sc * h;
            alo += sc * l;
            mh += mn * x.sh(G);
            ml += mn * x.sl(G);
        }
    }
    const float a = fmaf(256.f, (float)ah, (float)alo);
    const float m = fmaf(256.f, (float)mh, (float)ml);
    return x.s * (h2f(hd.x) * a - h2f(hd.x >> 16) * m);
}

// Q6_K: 2-byte aligned blocks; 24 shared loads per lane.
__device__ __forceinline__ float qdot_q6k(const uint8_t* bp, int o, const XLane& x) {
    const uint8_t* al = reinterpret_cast<const uint8_t*>((uintptr_t)bp & ~(uintptr_t)3);
    const int sh = 8 * (int)((uintptr_t)bp & 3);
    const uint2 ha = lds64_a2(al + 128 + 8 * o, sh), hb = lds64_a2(al + 160 + 8 * o, sh);
    const uint32_t v0 = lds32(al + 192), v1 = lds32(al + 196), v2 = lds32(al + 200),
                   v3 = lds32(al + 204), v4 = lds32(al + 208);
    const uint32_t sw[4] = {__funnelshift_r(v0, v1, sh), __funnelshift_r(v1, v2, sh),
                            __funnelshift_r(v2, v3, sh), __funnelshift_r(v3, v4, sh)};
    const float d = h2f(__funnelshift_r(v4, v4, sh));
    const int jo = o >> 1;
    int ah = 0, alo = 0;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint2 w = lds64_a2(al + 64 * (G >> 2) + 32 * (G & 1) + 8 * o, sh);
        const int ns = 4 * ((G >> 1) & 1), hs = 2 * (G & 3);
        const uint32_t h0 = G < 4 ? ha.x : hb.x, h1 = G < 4 ? ha.y : hb.y;
        const uint32_t u0 = ((w.x >> ns) & 0x0F0F0F0Fu) | (((h0 >> hs) & 0x03030303u) << 4);
        const uint32_t u1 = ((w.y >> ns) & 0x0F0F0F0Fu) | (((h1 >> hs) & 0x03030303u) << 4);
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(u1, xh.y, dp4(u0, xh.x, -32 * x.sh(G)));
        const int l = dp4(u1, xl.y, dp4(u0, xl.x, -32 * x.sl(G)));
        const int si = 2 * G + jo;  // int8 scale byte si of bytes 192..207
        const int s8 = sbyte(sw[si >> 2], si & 3);
        ah += s8 * h;
        alo += s8 * l;
    }
    return d * x.s * fmaf(256.f, (float)ah, (float)alo);
}

// Q8_0: bp points at 8 consecutive 34-byte blocks (256 values, 16-byte
// aligned); block G starts at 34*G (2-byte aligned).
__device__ __forceinline__ float qdot_q8_0(const uint8_t* bp, int o, const XLane& x) {
    float acc = 0.f;
#pragma unroll
    for (int G = 0; G < 8; ++G) {
        const uint8_t* qb = bp + 34 * G;
        // bytes qb[0..1] = d, qb[2 + 8o .. 10 + 8o) = quants
        const uint8_t* al = reinterpret_cast<const uint8_t*>((uintptr_t)(qb + 2 + 8 * o) & ~(uintptr_t)3);
        const int sh = 8 * (int)((uintptr_t)(qb + 2 + 8 * o) & 3);
        const uint2 q = lds64_a2(al, sh);
        const float dg = h2f(*reinterpret_cast<const uint16_t*>(qb));
        const uint2 xh = x.h2(G), xl = x.l2(G);
        const int h = dp4(q.y, xh.y, dp4(q.x, xh.x, 0));
        const int l = dp4(q.y, xl.y, dp4(q.x, xl.x, 0));
        acc = fmaf(dg, fmaf(256.f, (float)h, (float)l), acc);
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

// Out-of-line dots of one lane's pair (b, o) of one or two rows with the
// activation codes at `codes` (a QVec of n values), the codes loaded
// inside.  Each kernel that calls these holds one copy of each decoder, so
// a step that runs every phase once stays small in the instruction cache
// (an inlined decoder at every call site made the single-token decode
// kernel's step ~200 KB of code, fetched again from L2 every step).
template <int T>
static __device__ __noinline__ float2 qdot2_rows(int rt0, const uint8_t* row0, int rt1,
                                                 const uint8_t* row1, uint8_t* codes, int n,
                                                 int b, int o) {
    XLane x;
    load_xlane(x, qvec_at(codes, n), b, o);
    return make_float2(qdot_t<T>(rt0, row0, b, o, x), qdot_t<T>(rt1, row1, b, o, x));
}

template <int T>
static __device__ __noinline__ float qdot1_row(int rt, const uint8_t* row, uint8_t* codes, int n,
                                               int b, int o) {
    XLane x;
    load_xlane(x, qvec_at(codes, n), b, o);
    return qdot_t<T>(rt, row, b, o, x);
}

// Sum over the `lpr` consecutive lanes of a row group (lpr a power of two).
__device__ __forceinline__ float group_sum(float v, int lpr) {
    for (int off = lpr >> 1; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    return v;
}

}  // namespace moeb200
