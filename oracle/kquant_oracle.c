/*
 * kquant_oracle.c -- CPU restatement of the reference K-quant hot path.
 *
 * TEST INFRASTRUCTURE ONLY (see kquant_oracle.h).  The product library never
 * links or calls this file; it is the checker the GPU kernels are compared
 * against, and the scalar CPU port timed as a baseline.
 *
 * Every function names the reference code it restates (paths relative to the
 * reference project root).  The arithmetic order is kept exactly:
 *   - dequantised values are computed as (d*scale)*q [- dmin*min] with one
 *     rounding per operation and no fused multiply-add, as in the reference
 *     decoders and in gguf.quants;
 *   - dot products accumulate into eight lanes, lane = column % 8, with one
 *     fused multiply-add per weight, then sum the lanes 0..7 into a zero
 *     start value, as the reference's AVX2 __m256 accumulator does.
 * Build with -ffp-contract=off so the compiler adds no contractions.
 */
#include "kquant_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------ half floats */

/* IEEE binary16 -> binary32, exact for every input.
   Restates f16_to_f32 (cpp/dequant_k.cpp:49-77). */
float kq_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h >> 15) << 31;
    const uint32_t e = (h >> 10) & 31u;
    const uint32_t m = h & 1023u;
    uint32_t bits;
    if (e == 31u) {
        bits = sign | 0x7F800000u | (m << 13);
    } else if (e == 0u) {
        /* zero or subnormal: m * 2^-24 is exact in binary32 */
        const float v = ldexpf((float)m, -24);
        return sign ? -v : v;
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

/* binary32 -> binary16, round to nearest even, subnormals kept.
   Restates f32_to_f16 (cpp/dequant_k.cpp:79-111) and the F16C conversion
   with rounding control 0 used by cvt_f32_to_f16 (:124-136) and round16
   (cpp/moe_quant_dot.cpp:8-10). */
uint16_t kq_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
    const uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) {                       /* inf / nan */
        if (ax == 0x7F800000u) return (uint16_t)(sign | 0x7C00u);
        return (uint16_t)(sign | 0x7E00u | ((ax >> 13) & 0x3FFu));
    }
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  /* >= 65520 */
    if (ax < 0x38800000u) {                        /* below 2^-14 */
        float v;
        memcpy(&v, &ax, 4);
        /* v * 2^24 is exact; the integer part is the subnormal code
           (1024 rolls over into the smallest normal, which is correct). */
        const uint32_t q = (uint32_t)nearbyintf(v * 16777216.0f);
        return (uint16_t)(sign | q);
    }
    const uint32_t e = (ax >> 23) - 112u;
    uint32_t h = (e << 10) | ((ax & 0x7FFFFFu) >> 13);
    const uint32_t rem = ax & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)(sign | h);
}

float kq_round16(float f) { return kq_f16_to_f32(kq_f32_to_f16(f)); }

/* ------------------------------------------------------------ block sizes */

/* block_size_of / bytes_per_block (cpp/dequant_k.cpp:302-322). */
int kq_block_size(int type) {
    switch (type) {
        case KQ_Q8_0: return 32;
        case KQ_Q3_K: case KQ_Q4_K: case KQ_Q5_K: case KQ_Q6_K: return 256;
        default: return 0;
    }
}

int kq_block_bytes(int type) {
    switch (type) {
        case KQ_Q8_0: return 34;
        case KQ_Q3_K: return 110;
        case KQ_Q4_K: return 144;
        case KQ_Q5_K: return 176;
        case KQ_Q6_K: return 210;
        default: return 0;
    }
}

static float rd_f16(const uint8_t* p) {
    return kq_f16_to_f32((uint16_t)(p[0] | (p[1] << 8)));
}

/* ------------------------------------------------------------ decoders */

/* Q8_0: 34 bytes = f16 d, int8 q[32]; y = q * d.
   Restates dequant_q8_0 (cpp/dequant_k.cpp:146-154). */
static void dq_q8_0(const uint8_t* b, float* y) {
    const float d = rd_f16(b);
    for (int j = 0; j < 32; ++j) y[j] = (float)(int8_t)b[2 + j] * d;
}

/* Six-bit scale/min pairs shared by Q4_K and Q5_K.
   Restates unpack_scale_min_k4 (cpp/dequant_k.cpp:166-175). */
static void k4_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

/* Q4_K: 144 bytes = f16 d, f16 dmin, 12 scale bytes, 128 nibble bytes.
   Values 64g..64g+31 are the low nibbles of bytes 16+32g.., values
   64g+32..64g+63 the high nibbles; y = (d*sc)*q - dmin*mn.
   Restates dequant_q4_k (cpp/dequant_k.cpp:182-206). */
static void dq_q4_k(const uint8_t* b, float* y) {
    const float d = rd_f16(b), dmin = rd_f16(b + 2);
    for (int i = 0; i < 256; ++i) {
        const int j = i >> 5;
        int sc, mn;
        k4_scale_min(b + 4, j, &sc, &mn);
        const uint8_t byte = b[16 + (i >> 6) * 32 + (i & 31)];
        const int q = (j & 1) ? (byte >> 4) : (byte & 15);
        const float d1 = d * (float)sc;
        const float m1 = dmin * (float)mn;
        y[i] = d1 * (float)q - m1;
    }
}

/* Q5_K: 176 bytes = f16 d, f16 dmin, 12 scale bytes, qh[32], qs[128].
   Low four bits as Q4_K (from byte 48), bit 4 is bit i/32 of qh[i%32];
   y = (d*sc)*q - dmin*mn.
   Restates dequant_q5_k (cpp/dequant_k.cpp:221-240) with the byte/shift
   tables of cpp/dequant_k_tables.h:29-36 written as their closed form. */
static void dq_q5_k(const uint8_t* b, float* y) {
    const float d = rd_f16(b), dmin = rd_f16(b + 2);
    for (int i = 0; i < 256; ++i) {
        const int j = i >> 5;
        int sc, mn;
        k4_scale_min(b + 4, j, &sc, &mn);
        const uint8_t byte = b[48 + (i >> 6) * 32 + (i & 31)];
        const int lo = (j & 1) ? (byte >> 4) : (byte & 15);
        const int hi = (b[16 + (i & 31)] >> j) & 1;
        const int q = lo | (hi << 4);
        y[i] = d * (float)sc * (float)q - dmin * (float)mn;
    }
}

/* Q6_K: 210 bytes = ql[128], qh[64], int8 scales[16], f16 d.
   q = (ql nibble | qh 2 bits << 4) - 32; y = (d*scale[i/16])*q.
   Restates dequant_q6_k (cpp/dequant_k.cpp:254-268) with the tables of
   cpp/dequant_k_tables.h:24-27 written as their closed form. */
static void dq_q6_k(const uint8_t* b, float* y) {
    const float d = rd_f16(b + 208);
    for (int i = 0; i < 256; ++i) {
        const int lo = (b[(i >> 7) * 64 + (i & 63)] >> (((i >> 6) & 1) * 4)) & 15;
        const int hi = (b[128 + (i >> 7) * 32 + (i & 31)] >> (((i >> 5) & 3) * 2)) & 3;
        const int q = (lo | (hi << 4)) - 32;
        y[i] = d * (float)(int8_t)b[192 + (i >> 4)] * (float)q;
    }
}

/* Q3_K: 110 bytes = hmask[32], qs[64], 12 scale bytes, f16 d at 108.
   q = ((qs byte >> 2*((i/32)%4)) & 3) - 4*(1 - hmask bit i/32);
   scale j = (low4 | high2 << 4) - 32; y = (d*scale[i/16])*q.
   Restates dequant_q3_k (cpp/dequant_k.cpp:278-298) with the tables of
   cpp/dequant_k_tables.h:19-22 written as their closed form. */
static void dq_q3_k(const uint8_t* b, float* y) {
    const uint8_t* s = b + 96;
    const float d = rd_f16(b + 108);
    int scale[16];
    for (int j = 0; j < 16; ++j) {
        const int low4 = (j < 8) ? (s[j] & 15) : (s[j - 8] >> 4);
        const int high2 = (s[8 + (j & 3)] >> (2 * (j >> 2))) & 3;
        scale[j] = (low4 | (high2 << 4)) - 32;
    }
    for (int i = 0; i < 256; ++i) {
        const int ql = (b[32 + (i >> 7) * 32 + (i & 31)] >> (2 * ((i >> 5) & 3))) & 3;
        const int hbit = (b[i & 31] >> (i >> 5)) & 1;
        const int q = ql - ((hbit ^ 1) << 2);
        y[i] = d * (float)scale[i >> 4] * (float)q;
    }
}

int kq_dequant_block(int type, const uint8_t* blk, float* out) {
    switch (type) {
        case KQ_Q8_0: dq_q8_0(blk, out); return 0;
        case KQ_Q3_K: dq_q3_k(blk, out); return 0;
        case KQ_Q4_K: dq_q4_k(blk, out); return 0;
        case KQ_Q5_K: dq_q5_k(blk, out); return 0;
        case KQ_Q6_K: dq_q6_k(blk, out); return 0;
        default: return -1;
    }
}

/* Restates the dequant_k export (cpp/dequant_k.cpp:350-394): -1 on an
   unknown type, a null pointer, n <= 0 or n not a whole number of blocks;
   f32 output, or binary16 rounded to nearest even when want_f16 != 0. */
int kq_dequant(int type, const uint8_t* src, void* dst, int64_t n, int want_f16) {
    const int bs = kq_block_size(type), pb = kq_block_bytes(type);
    if (bs == 0 || src == NULL || dst == NULL) return -1;
    if (n <= 0 || n % bs != 0) return -1;
    float tmp[256];
    for (int64_t b = 0; b < n / bs; ++b) {
        kq_dequant_block(type, src + b * pb, tmp);
        if (want_f16) {
            uint16_t* o = (uint16_t*)dst + b * bs;
            for (int j = 0; j < bs; ++j) o[j] = kq_f32_to_f16(tmp[j]);
        } else {
            memcpy((float*)dst + b * bs, tmp, sizeof(float) * (size_t)bs);
        }
    }
    return 0;
}

/* Restates quant_dot (cpp/moe_quant_dot.cpp:143-169) and its fused Q3_K /
   Q6_K variants (:25-139): weight j of each block is the dequantised value
   (optionally rounded to binary16), folded into lane (column % 8) with a
   fused multiply-add in column order; the lanes are then summed 0..7. */
float kq_quant_dot(int type, const uint8_t* row, const float* x, int columns,
                   int round_weights) {
    const int bs = kq_block_size(type), pb = kq_block_bytes(type);
    float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float w[256];
    for (int off = 0; off < columns; off += bs, row += pb) {
        kq_dequant_block(type, row, w);
        for (int j = 0; j < bs; ++j) {
            const float wj = round_weights ? kq_round16(w[j]) : w[j];
            lanes[j & 7] = fmaf(wj, x[off + j], lanes[j & 7]);
        }
    }
    float r = 0.0f;
    for (int l = 0; l < 8; ++l) r += lanes[l];
    return r;
}

/* Restates the moe_quant_expert export (cpp/moe_quant_dot.cpp:171-214):
   validation order and status codes (-1 arguments, -2 type or column
   multiple, -3 byte count, -4 non-finite output, -5 allocation), and in
   fp16_graph mode the seven binary16 rounding points (x, every weight, g, u,
   sigmoid, silu, the activation, the output). */
int kq_expert(int gate_type, const uint8_t* gate, int64_t gate_bytes,
              int up_type, const uint8_t* up, int64_t up_bytes,
              int down_type, const uint8_t* down, int64_t down_bytes,
              const float* input, int hidden, int intermediate, float* output,
              int fp16_graph) {
    const int types[3] = {gate_type, up_type, down_type};
    const int cols[3] = {hidden, hidden, intermediate};
    const int rows[3] = {intermediate, intermediate, hidden};
    const int64_t sizes[3] = {gate_bytes, up_bytes, down_bytes};
    if (!gate || !up || !down || !input || !output || hidden <= 0 ||
        intermediate <= 0 || hidden > 65536 || intermediate > 65536 ||
        (fp16_graph != 0 && fp16_graph != 1))
        return -1;
    for (int i = 0; i < 3; ++i) {
        const int bs = kq_block_size(types[i]);
        if (!bs || cols[i] % bs) return -2;
        const int64_t expected = (int64_t)rows[i] * (cols[i] / bs) * kq_block_bytes(types[i]);
        if (sizes[i] != expected) return -3;
    }
    float* x = (float*)malloc(sizeof(float) * (size_t)hidden);
    float* act = (float*)malloc(sizeof(float) * (size_t)intermediate);
    if (!x || !act) { free(x); free(act); return -5; }
    for (int i = 0; i < hidden; ++i) x[i] = fp16_graph ? kq_round16(input[i]) : input[i];
    const int64_t gr = (int64_t)(hidden / kq_block_size(gate_type)) * kq_block_bytes(gate_type);
    const int64_t ur = (int64_t)(hidden / kq_block_size(up_type)) * kq_block_bytes(up_type);
    const int64_t dr = (int64_t)(intermediate / kq_block_size(down_type)) * kq_block_bytes(down_type);
    for (int r = 0; r < intermediate; ++r) {
        float g = kq_quant_dot(gate_type, gate + r * gr, x, hidden, fp16_graph);
        float u = kq_quant_dot(up_type, up + r * ur, x, hidden, fp16_graph);
        if (fp16_graph) { g = kq_round16(g); u = kq_round16(u); }
        float sig = 1.0f / (1.0f + expf(-g));
        if (fp16_graph) sig = kq_round16(sig);
        float silu = g * sig;
        if (fp16_graph) silu = kq_round16(silu);
        const float a = silu * u;
        act[r] = fp16_graph ? kq_round16(a) : a;
    }
    int status = 0;
    for (int r = 0; r < hidden; ++r) {
        const float y = kq_quant_dot(down_type, down + r * dr, act, intermediate, fp16_graph);
        output[r] = fp16_graph ? kq_round16(y) : y;
        if (!isfinite(output[r])) { status = -4; break; }
    }
    free(x);
    free(act);
    return status;
}

/* ------------------------------------------------------- DeltaNet step */

/* Sum of an eight-lane accumulator, lanes 0..7 into a zero start value
   (sum8, cpp/moe_delta.cpp:10-16). */
static float kq_sum8(const float lanes[8]) {
    float s = 0.0f;
    for (int l = 0; l < 8; ++l) s += lanes[l];
    return s;
}

/* Restates moe_delta_heads (cpp/moe_delta.cpp:18-69).  Per head h:
 *   decay = exp((double)gate[h]);
 * per state row r (key_dim values):
 *   row[j] <- (float)((double)row[j] * decay)                (stored)
 *   kv     = sum_j row[j] * k[h][j]  -- eight lanes (lane = j % 8) over the
 *            whole groups of eight, summed lanes 0..7, then the tail j in
 *            order; each term one multiply then one add, no fusing
 *   delta  = beta[h] * (v[h][r] - kv)
 *   row[j] <- row[j] + delta * k[h][j]                       (stored)
 *   out    = sum_j row[j] * q[h][j]  -- same lane order as kv
 * A non-finite out returns -2 at once: this row and every row before it are
 * already updated, its output and every later row are untouched. */
int kq_delta_heads(float* state, const float* q, const float* k,
                   const float* v, const float* beta, const float* gate,
                   float* output, int heads, int key_dim, int value_dim) {
    if (!state || !q || !k || !v || !beta || !gate || !output ||
        heads < 1 || heads > 256 || key_dim < 1 || key_dim > 1024 ||
        value_dim < 1 || value_dim > 1024)
        return -1;
    const int whole = key_dim - key_dim % 8;
    for (int h = 0; h < heads; ++h) {
        const double decay = exp((double)gate[h]);
        const float* kh = k + (int64_t)h * key_dim;
        const float* qh = q + (int64_t)h * key_dim;
        for (int r = 0; r < value_dim; ++r) {
            float* row = state + ((int64_t)h * value_dim + r) * key_dim;
            float lanes[8] = {0, 0, 0, 0, 0, 0, 0, 0};
            int j = 0;
            for (; j < whole; ++j) {
                row[j] = (float)((double)row[j] * decay);
                const float p = row[j] * kh[j];
                lanes[j % 8] = lanes[j % 8] + p;
            }
            float kv = kq_sum8(lanes);
            for (; j < key_dim; ++j) {
                row[j] = (float)((double)row[j] * decay);
                const float p = row[j] * kh[j];
                kv = kv + p;
            }
            const float delta = beta[h] * (v[(int64_t)h * value_dim + r] - kv);
            for (int l = 0; l < 8; ++l) lanes[l] = 0.0f;
            for (j = 0; j < whole; ++j) {
                const float t = delta * kh[j];
                row[j] = row[j] + t;
                const float p = row[j] * qh[j];
                lanes[j % 8] = lanes[j % 8] + p;
            }
            float result = kq_sum8(lanes);
            for (; j < key_dim; ++j) {
                const float t = delta * kh[j];
                row[j] = row[j] + t;
                const float p = row[j] * qh[j];
                result = result + p;
            }
            if (!isfinite(result)) return -2;
            output[(int64_t)h * value_dim + r] = result;
        }
    }
    return 0;
}
