// prefill.cu -- many-token MoE layer on the tcgen05 tensor cores.
//
// Same layer as run_moe_sequence (reference src/flash_moe/moe_layer.py:110-195):
// route every token (fp32 router logits, top-k, float64 softmax), group the
// (token, slot) pairs by expert, run each expert's SwiGLU FFN over its group
// (the reference batches them through forward_batch, backend_ov.py:357-431),
// weight the outputs by the routing weights and add the sigmoid-gated shared
// expert (shared_expert.py:200-219).
//
// Arithmetic.  The expert weights are dequantised to fp16 in shared memory
// with the same value the reference's f16 dequantisation gives
// (cpp/dequant_k.cpp:324-394: the fp32 value of dequant_k rounded to nearest
// even), and the GEMMs run as tcgen05.mma kind::f16 with fp32 accumulation
// in tensor memory.  The activations enter as fp16 scaled per token by a
// power of two (exact; undone in the epilogue).  The SwiGLU product is
// formed in fp32 and stored as fp16 for the down projection.  The router
// logits use the same MMAs on an fp16 hi/lo split of x and of the router
// rows (three products: hi.hi + lo.hi + hi.lo, ~2^-22 relative), each
// scaled by a power of two, so they stay within ~1e-6 of fp32.
//
// Kernels of one call (one stream):
//   k_pf_prep_x      per token: power-of-two scale, fp16 hi/lo, shared-gate
//                    sigmoid, zero the output row
//   k_pf_prep_router per router row: power-of-two scale, fp16 hi/lo
//                    (k_pf_router_small instead, fp32 on the CUDA cores, for
//                    at most 128 tokens)
//   k_pf_gemm<ROUTER> logits = x . router^T (+ bias)
//   k_pf_topk        per token (one warp): top-k + softmax (topk.cuh), pair
//                    counts per held expert (done by k_pf_router_small for
//                    few tokens and at most 256 experts)
//   k_pf_pairs       per pair (one warp): its slot in the held expert's pair
//                    list (expert offsets by a prefix sum of the counts, a
//                    slot cursor per expert) and the copy of its x row there
//                    (contiguous B rows per expert)
//   k_pf_gemm<GATEUP> act = silu(x Wg^T) * (x Wu^T) per pair, fp16
//   k_pf_gemm<DOWN>  y[token] += w * (act Wd^T) per pair (fp32 reductions)
//
// The GEMM kernel is persistent (one CTA per SM, 480 threads) and
// warp-specialised:
//   warps 0-3  epilogue: TMEM -> registers -> global (lane = tile row)
//   warp 4     TMEM allocation; lane 0 issues the MMAs
//   warp 5     TMA producer of B, the token rows of the unit's pairs: the
//              permuted x rows (gate/up) or the act rows (down), 2-D boxes
//              of 128 and 16 rows
//   warps 6-13 dequantisation: raw blocks -> fp16 K-major 128B-swizzled A
//   warp 14    TMA producer of the packed weight rows (raw bytes, 2-D boxes),
//              up to four 256-value groups ahead
// A unit of work is one expert x 128 weight rows x up to 256 pairs (tokens)
// over the whole K; the K loop runs in stages of 64 values.  Mbarriers
// connect the roles; every wait is bounded and a timeout sets the error
// word and ends the kernel.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <math.h>

#include <cstdlib>
#include <mutex>
#include <utility>

#include "launch.h"
#include "topk.cuh"
#include "umma.cuh"

namespace moeb200 {

enum PfMode { PF_ROUTER = 0, PF_GATEUP = 1, PF_DOWN = 2 };

constexpr int kPfThreads = 480;
constexpr int kPfEpiWarps = 4;
constexpr int kPfMmaWarp = 4;
constexpr int kPfProdWarp = 5;
constexpr int kPfDqWarp0 = 6;
constexpr int kPfRawWarp = 14;
constexpr int kPfDqThreads = 256;
constexpr int kPfMaxN = 256;
constexpr int kPfRouterN = 256;     // ROUTER: tokens per unit (MMA N)
constexpr int kPfRouterChunks = 8;  // ROUTER: K chunks (units per token tile and row tile)
constexpr uint32_t kPfPolls = 1u << 22;
constexpr int kPfMaxExperts = 1024;


// Raw group of a block format: values, bytes and the TMA box width (the
// smallest odd multiple of 16 bytes covering the group at any 16-byte
// misalignment; odd so that rows of the box fall in distinct bank groups).
__host__ __device__ constexpr int pf_gv(int t) { return t == Q8_0 ? 128 : 256; }
__host__ __device__ constexpr int pf_gb(int t) {
    return t == Q8_0 ? 136 : t == Q3_K ? 110 : t == Q4_K ? 144 : t == Q5_K ? 176 : 210;
}
__host__ __device__ constexpr int pf_w(int t) {
    return t == Q5_K ? 176 : t == Q6_K ? 240 : 144;
}

struct PfSide {
    int type;   // block format of the gate (or down) matrix
    int type2;  // block format of the up matrix (same raw group size)
    int rows;   // rows of one expert matrix
    int K;      // columns
};

struct __align__(64) PfParams {
    CUtensorMap wmap[2][2];  // [routed, shared][gate or down, up]: raw weight bytes
    CUtensorMap bmap[2][2];  // [routed, shared][box of 128 rows, of 16 rows]: B rows
                             // (gate/up: x in pair order / x; down: act)
    CUtensorMap rbmap[2];    // ROUTER B: fp16 x hi, lo (boxes of 16 rows)
    CUtensorMap rmap[2];     // ROUTER A: router rows hi, lo
    PfSide side[2];
    int n_routed;            // routed experts held (units on side 0)
    int has_shared;
    int T, H, E, Imax;
    int segs;                // ROUTER: K segments (2: x exact in fp16; 3)
    int rchunks;             // ROUTER: K chunks of the segs * H / 64 stages
    float* rpart;            // ROUTER: [rchunks x T x E] scaled partial logits
    int stages, raw_slots;
    uint32_t stage_bytes, a_bytes, raw_slot_bytes;
    const int32_t* counts;   // [n_routed] pairs per held expert
    const int32_t* pair_tok; // [pairs] token of each pair, expert-major
    const float* pair_w;     // [pairs] routing weight of each pair
    const float* sg;         // [T] shared-expert gate
    const float* xs_inv;     // [T] 2^-k of the token scale
    const float* rs_inv;     // [E] 2^-k of the router row scale
    const float* bias;       // [E] or null
    __half* act;             // [(pairs + T) x Imax]
    float* y;                // [T x H]
    float* logits;           // [T x E]
    uint32_t* err;
    uint64_t* trace;         // null, or 32 slots per CTA: per-role wait cycles
};

// ---------------------------------------------------------------------------
// small helpers

__device__ __forceinline__ __half2 u2h2(uint32_t u) {
    __half2 h;
    memcpy(&h, &u, 4);
    return h;
}
__device__ __forceinline__ uint32_t h22u(__half2 h) {
    uint32_t u;
    memcpy(&u, &h, 4);
    return u;
}
__device__ __forceinline__ uint32_t f2h2u(float a, float b) {
    return h22u(__floats2half2_rn(a, b));
}
__device__ __forceinline__ float h16f(uint32_t bits) {
    return __half2float(__ushort_as_half((unsigned short)bits));
}

template <int NW>
__device__ __forceinline__ uint32_t nbyte(const uint32_t (&w)[NW], int k) {
    return (w[k >> 2] >> (8 * (k & 3))) & 0xFFu;
}
template <int NW>
__device__ __forceinline__ uint32_t nhalf(const uint32_t (&w)[NW], int k) {
    return (w[k >> 2] >> (8 * (k & 3))) & 0xFFFFu;  // k even
}
// 4 bytes at byte offset k (k even)
template <int NW>
__device__ __forceinline__ uint32_t nword(const uint32_t (&w)[NW], int k) {
    return (k & 3) ? __funnelshift_r(w[k >> 2], w[(k >> 2) + 1], 16) : w[k >> 2];
}

// fp32 value of the byte b (0..255) plus 2^23
__device__ __forceinline__ float magic_f(uint32_t word, int k) {
    return __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540u | (uint32_t)k));
}

// Position in a ring of n mbarrier-guarded slots: the slot index in the low
// 16 bits, the phase parity in bit 16 (no division by the run-time ring size
// on the per-stage path).
__device__ __forceinline__ uint32_t ring_next(uint32_t it, uint32_t n) {
    return ((it & 0xFFFFu) + 1u == n) ? ((it & 0x10000u) ^ 0x10000u) : it + 1u;
}

__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                        uint32_t* err) {
    for (uint32_t i = 0; i < kPfPolls; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31u) == 31u && *abort) return false;
    }
    atomicCAS(err, 0u, (uint32_t)ST_TIMEOUT);
    *abort = 1;
    return false;
}

// pf_wait that adds the cycles it spent to *acc (when acc is not null)
__device__ __forceinline__ bool pf_wait_t(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint32_t* err, uint64_t* acc) {
    if (!acc) return pf_wait(bar, parity, abort, err);
    const uint64_t t0 = clock64();
    const bool ok = pf_wait(bar, parity, abort, err);
    *acc += clock64() - t0;
    return ok;
}

// ---------------------------------------------------------------------------
// dequantisation of one raw group row (normalised words: block-relative
// little-endian words) into fp16 chunks of 8 values (one 16-byte chunk of a
// K-major row).  Chunk c of stage s covers group values 64 s + 8 c .. +7.
// Every value equals the reference's fp32 dequantisation rounded to fp16.

template <int T>
struct PfNW {
    static constexpr int n = (pf_gb(T) + 3) / 4;
};

// Q3_K: (d * sc) * q with |sc * q| <= 128, so q * sc is exact in fp16 and a
// single fp16 multiply by d rounds the exact product, like fp32 then fp16.
template <int S, int C>
__device__ __forceinline__ uint4 dq_chunk_q3(const uint32_t (&w)[28]) {
    constexpr int c4 = C & 3, sub = 2 * S + (C >> 2);  // i/32 of the chunk
    constexpr int qw = (32 + 32 * (S >> 1) + 8 * c4) >> 2;
    constexpr int sh = 2 * (sub & 3);
    constexpr int j = 4 * S + (C >> 1);  // scale index
    const uint32_t lo4 = (j < 8) ? (nbyte(w, 96 + j) & 15u) : (nbyte(w, 96 + j - 8) >> 4);
    const uint32_t hi2 = (nbyte(w, 104 + (j & 3)) >> (2 * (j >> 2))) & 3u;
    const uint32_t sv = lo4 | (hi2 << 4);  // sc + 32
    const __half2 sc2 = __hsub2(u2h2(0x64006400u | sv | (sv << 16)), __float2half2_rn(1056.f));
    const uint32_t db = nhalf(w, 108);
    const __half2 d2 = u2h2(db | (db << 16));
    const __half2 k1028 = __float2half2_rn(1028.f);
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t qs = w[qw + h], hm = w[2 * c4 + h];
        const uint32_t hb = (sub >= 2 ? (hm >> (sub - 2)) : (hm << (2 - sub))) & 0x04040404u;
        const uint32_t nb = ((qs >> sh) & 0x03030303u) | hb;  // q + 4 per byte
        const __half2 q01 = __hsub2(u2h2(__byte_perm(nb, 0x64646464u, 0x4140u)), k1028);
        const __half2 q23 = __hsub2(u2h2(__byte_perm(nb, 0x64646464u, 0x4342u)), k1028);
        o[2 * h] = h22u(__hmul2(__hmul2(q01, sc2), d2));
        o[2 * h + 1] = h22u(__hmul2(__hmul2(q23, sc2), d2));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// six-bit (scale, min) pair j of Q4_K/Q5_K from the 12 bytes at 4
template <int NW>
__device__ __forceinline__ void k4sm(const uint32_t (&w)[NW], int j, uint32_t& sc, uint32_t& mn) {
    if (j < 4) {
        sc = nbyte(w, 4 + j) & 63u;
        mn = nbyte(w, 8 + j) & 63u;
    } else {
        sc = (nbyte(w, 8 + j) & 15u) | ((nbyte(w, j) >> 6) << 4);
        mn = (nbyte(w, 8 + j) >> 4) | ((nbyte(w, 4 + j) >> 6) << 4);
    }
}

// Q4_K / Q5_K: fma(d*sc, q, -dmin*m) in fp32 (d*sc*q is exact, so the fma
// rounds like the reference's multiply then subtract), then fp16.
template <int T, int S, int C, int NW>
__device__ __forceinline__ uint4 dq_chunk_q45(const uint32_t (&w)[NW]) {
    constexpr int c4 = C & 3, j = 2 * S + (C >> 2);
    constexpr int qoff = (T == Q4_K ? 16 : 48) + 32 * S + 8 * c4;
    uint32_t sc, mn;
    k4sm(w, j, sc, mn);
    const float dsc = __fmul_rn(h16f(nhalf(w, 0)), (float)sc);
    const float dm = __fmul_rn(h16f(nhalf(w, 2)), (float)mn);
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        uint32_t nb = (w[(qoff >> 2) + h] >> (4 * (C >> 2))) & 0x0F0F0F0Fu;
        if (T == Q5_K) nb |= ((w[((16 + 8 * c4) >> 2) + h] >> j) & 0x01010101u) << 4;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = fmaf(dsc, magic_f(nb, k) - 8388608.f, -dm);
        o[2 * h] = f2h2u(v[0], v[1]);
        o[2 * h + 1] = f2h2u(v[2], v[3]);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Q6_K: (d*sc) * (q - 32) in fp32, then fp16.
template <int S, int C>
__device__ __forceinline__ uint4 dq_chunk_q6(const uint32_t (&w)[53]) {
    constexpr int c4 = C & 3, sub = 2 * S + (C >> 2);
    constexpr int lw = (64 * (S >> 1) + 8 * C) >> 2;
    constexpr int hw = (128 + 32 * (S >> 1) + 8 * c4) >> 2;
    constexpr int j = 4 * S + (C >> 1);
    const float ds = __fmul_rn(h16f(nhalf(w, 208)), (float)(int8_t)nbyte(w, 192 + j));
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t nb = ((w[lw + h] >> (4 * (S & 1))) & 0x0F0F0F0Fu) |
                            (((w[hw + h] >> (2 * (sub & 3))) & 0x03030303u) << 4);
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = __fmul_rn(ds, magic_f(nb, k) - 8388640.f);
        o[2 * h] = f2h2u(v[0], v[1]);
        o[2 * h + 1] = f2h2u(v[2], v[3]);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

// Q8_0 (group of four 34-byte blocks): q * d, exact in fp16 arithmetic.
template <int S, int C>
__device__ __forceinline__ uint4 dq_chunk_q8(const uint32_t (&w)[34]) {
    constexpr int blk = 2 * S + (C >> 2);
    constexpr int qo = 34 * blk + 2 + 8 * (C & 3);
    const uint32_t db = nhalf(w, 34 * blk);
    const __half2 d2 = u2h2(db | (db << 16));
    const __half2 k1152 = __float2half2_rn(1152.f);
    uint32_t o[4];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const uint32_t nb = nword(w, qo + 4 * h) ^ 0x80808080u;  // q + 128 per byte
        const __half2 q01 = __hsub2(u2h2(__byte_perm(nb, 0x64646464u, 0x4140u)), k1152);
        const __half2 q23 = __hsub2(u2h2(__byte_perm(nb, 0x64646464u, 0x4342u)), k1152);
        o[2 * h] = h22u(__hmul2(q01, d2));
        o[2 * h + 1] = h22u(__hmul2(q23, d2));
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int T, int S, int C, int NW>
__device__ __forceinline__ uint4 dq_chunk(const uint32_t (&w)[NW]) {
    if constexpr (T == Q3_K) return dq_chunk_q3<S, C>(w);
    else if constexpr (T == Q4_K || T == Q5_K) return dq_chunk_q45<T, S, C>(w);
    else if constexpr (T == Q6_K) return dq_chunk_q6<S, C>(w);
    else return dq_chunk_q8<S, C>(w);
}

// ---------------------------------------------------------------------------
// unit enumeration shared by all roles
//
// A GATEUP tile holds 64 gate rows and the same 64 up rows, interleaved in
// groups of eight: tile row r is row j = 8 (r / 16) + r % 8 of the gate
// (m = (r / 8) % 2 == 0) or of the up matrix (m == 1).  Lanes l and l ^ 8 of
// an epilogue warp therefore hold the gate and the up value of one
// intermediate row.  DOWN and ROUTER tiles are 128 consecutive rows.

__host__ __device__ constexpr int pf_tile_rows(int mode) { return mode == PF_GATEUP ? 64 : 128; }

struct PfShared {
    int n_units;
    int units_r;     // routed units
    int rt_r, rt_s;  // row tiles per routed / shared column tile
    int pairs;       // routed pairs in total
    int ntiles_r;
};

struct PfUnit {
    int side;  // 0 routed, 1 shared
    int e;     // held expert (routed)
    int n;     // valid columns (pairs)
    int rt;    // row tile
    int prow;  // first pair row (act rows for the shared side start after the routed)
    int tok0;  // shared / router: first token
    int kc;    // router: K chunk
};

template <int MODE>
__device__ __forceinline__ PfUnit pf_unit(const PfParams& p, const PfShared& sh,
                                          const int* s_tfirst, const int* s_poff, int u) {
    PfUnit r;
    if (MODE == PF_ROUTER) {
        const int rt_n = (p.E + 127) / 128, tt_n = (p.T + kPfRouterN - 1) / kPfRouterN;
        r.side = 0;
        r.e = 0;
        r.rt = u % rt_n;
        const int rest = u / rt_n;
        r.tok0 = (rest % tt_n) * kPfRouterN;
        r.kc = rest / tt_n;
        r.n = min(kPfRouterN, p.T - r.tok0);
        r.prow = r.tok0;
        return r;
    }
    if (u < sh.units_r) {
        const int tile = u / sh.rt_r;
        r.side = 0;
        r.rt = u % sh.rt_r;
        int lo = 0, hi = p.n_routed;  // last e with s_tfirst[e] <= tile
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (s_tfirst[mid] <= tile) lo = mid;
            else hi = mid;
        }
        r.e = lo;
        const int sub = tile - s_tfirst[lo];
        r.prow = s_poff[lo] + sub * kPfMaxN;
        r.n = min(kPfMaxN, s_poff[lo + 1] - r.prow);
        r.tok0 = 0;
    } else {
        const int v = u - sh.units_r;
        r.side = 1;
        r.e = 0;
        r.rt = v % sh.rt_s;
        r.tok0 = (v / sh.rt_s) * kPfMaxN;
        r.n = min(kPfMaxN, p.T - r.tok0);
        r.prow = sh.pairs + r.tok0;
    }
    return r;
}

// ---------------------------------------------------------------------------
// dequantisation role: one unit.  The thread owns tile row `trow` and writes
// chunks 4h..4h+3 of it per stage; its raw block row starts `rofs` bytes
// into the raw slot.

template <int T, int S>
__device__ __forceinline__ void dq_store(uint8_t* a, int trow, int h,
                                         const uint32_t (&w)[PfNW<T>::n]) {
    if (h == 0) {
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 0)) = dq_chunk<T, S, 0>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 1)) = dq_chunk<T, S, 1>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 2)) = dq_chunk<T, S, 2>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 3)) = dq_chunk<T, S, 3>(w);
    } else {
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 4)) = dq_chunk<T, S, 4>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 5)) = dq_chunk<T, S, 5>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 6)) = dq_chunk<T, S, 6>(w);
        *reinterpret_cast<uint4*>(a + sw128_offset(trow, 7)) = dq_chunk<T, S, 7>(w);
    }
}

template <int T, int MODE>
__device__ __forceinline__ bool dq_unit(const PfParams& p, const PfUnit& un, uint8_t* smem,
                                        uint64_t* full, uint64_t* empty, uint64_t* rfull,
                                        uint64_t* rempty, uint32_t& it_s, uint32_t& it_r,
                                        int trow, int h, uint32_t rofs, volatile int* abort,
                                        uint64_t* t_rfull, uint64_t* t_empty) {
    constexpr int GV = pf_gv(T), GB = pf_gb(T), W = pf_w(T), NSW = W / 4;
    constexpr int NW = PfNW<T>::n;
    constexpr int NST = GV / 64;
    const int groups = p.side[un.side].K / GV;
    const uint8_t* raw0 = smem + (size_t)p.stages * p.stage_bytes + rofs;
    for (int g = 0; g < groups; ++g) {
        const uint32_t slot = it_r & 0xFFFFu, rph = it_r >> 16;
        if (!pf_wait_t(&rfull[slot], rph, abort, p.err, t_rfull)) return false;
        const uint8_t* rr = raw0 + (size_t)slot * p.raw_slot_bytes;
        uint32_t src[NSW];
#pragma unroll
        for (int k = 0; k < W / 16; ++k) {
            const uint4 v = *reinterpret_cast<const uint4*>(rr + 16 * k);
            src[4 * k] = v.x;
            src[4 * k + 1] = v.y;
            src[4 * k + 2] = v.z;
            src[4 * k + 3] = v.w;
        }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&rempty[slot]);
        it_r = ring_next(it_r, p.raw_slots);
        // normalise: word i = bytes o + 4i .. o + 4i + 3 of the window
        const int o = (g * GB) & 15;
        uint32_t w[NW];
        if (GB % 16 == 0) {
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = src[i];
        } else {
            const int q = o >> 2;
            const uint32_t b = (uint32_t)(o & 3) * 8u;
            uint32_t t1[NSW];
#pragma unroll
            for (int i = 0; i < NSW; ++i) t1[i] = (q & 1) ? (i + 1 < NSW ? src[i + 1] : 0u) : src[i];
#pragma unroll
            for (int i = 0; i < NSW; ++i) src[i] = (q & 2) ? (i + 2 < NSW ? t1[i + 2] : 0u) : t1[i];
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(src[i], src[i + 1], b);
        }
        auto stage = [&](auto s_c) -> bool {
            const uint32_t st = it_s & 0xFFFFu, ph = it_s >> 16;
            if (!pf_wait_t(&empty[st], ph ^ 1u, abort, p.err, t_empty)) return false;
            dq_store<T, decltype(s_c)::value>(smem + (size_t)st * p.stage_bytes, trow, h, w);
            fence_async_smem();
            __syncwarp();
            if ((threadIdx.x & 31) == 0) mbar_arrive(&full[st]);
            it_s = ring_next(it_s, p.stages);
            return true;
        };
        if (!stage(std::integral_constant<int, 0>{})) return false;
        if (!stage(std::integral_constant<int, 1>{})) return false;
        if constexpr (NST == 4) {
            if (!stage(std::integral_constant<int, 2>{})) return false;
            if (!stage(std::integral_constant<int, 3>{})) return false;
        }
    }
    return true;
}

// y[0..3] += (a, b, c, d) as one vector reduction (16-byte aligned y)
__device__ __forceinline__ void red_add_v4(float* y, float a, float b, float c, float d) {
    asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(y), "f"(a), "f"(b),
                 "f"(c), "f"(d)
                 : "memory");
}

__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Barrier over the 128 epilogue threads that returns the OR of `pred`, so
// that they all leave their loop together.
__device__ __forceinline__ bool epi_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred)
        : "memory");
    return r != 0;
}

// ---------------------------------------------------------------------------
// the GEMM kernel

template <int MODE>
__global__ void __launch_bounds__(kPfThreads, 1) k_pf_gemm(const __grid_constant__ PfParams p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int S = p.stages, R = p.raw_slots;
    constexpr int NBUF = 2;  // accumulator buffers (256 columns each)
    const uint64_t t_start = clock64();
    uint64_t c0 = 0, c1 = 0;  // this role's wait cycles (traced lanes only)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * p.stage_bytes +
                                                 (size_t)R * p.raw_slot_bytes);
    uint64_t* empty = full + S;
    uint64_t* rfull = empty + S;
    uint64_t* rempty = rfull + R;
    uint64_t* acc_full = rempty + R;
    uint64_t* acc_empty = acc_full + 2;
    // (2 S + 2 R + 4) barriers of 8 bytes: s_tmem is 16-byte aligned, and
    // so is the transpose buffer 16 bytes after it (it takes 16-byte loads)
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acc_empty + 2);
    volatile int* s_abort = reinterpret_cast<volatile int*>(s_tmem + 1);
    float* s_tr = reinterpret_cast<float*>(s_tmem + 4);        // [4 warps][256] epilogue transpose
    int* s_ctok = reinterpret_cast<int*>(s_tr + 4 * 256);      // [256] column token
    float* s_cw = reinterpret_cast<float*>(s_ctok + kPfMaxN);  // [256] column scale / weight
    int* s_tfirst = reinterpret_cast<int*>(s_cw + kPfMaxN);
    int* s_poff = s_tfirst + (p.n_routed + 1);

    // --- set-up
    if (warp == kPfMmaWarp) tmem_alloc(s_tmem, 512);
    if (tid == 0) {
        // stage full: the B producer (its expect_tx arrival) and one arrival
        // per dequantisation warp
        const uint32_t fcount = (MODE == PF_ROUTER) ? 1u : 1u + kPfDqThreads / 32;
        for (int i = 0; i < S; ++i) {
            mbar_init(&full[i], fcount);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < R; ++i) {
            mbar_init(&rfull[i], 1);
            mbar_init(&rempty[i], kPfDqThreads / 32);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], kPfEpiWarps);
        }
        *s_abort = 0;
        mbar_fence_init();
    }
    PfShared sh{};
    if (MODE != PF_ROUTER && warp == 0) {
        // column tiles and pair offsets of the held experts (exclusive prefix sums)
        int carry_t = 0, carry_p = 0;
        for (int base = 0; base < p.n_routed; base += 32) {
            const int e = base + lane;
            const int c = e < p.n_routed ? p.counts[e] : 0;
            const int t0 = (c + kPfMaxN - 1) / kPfMaxN;
            int tl = t0, pc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, tl, o);
                const int b = __shfl_up_sync(0xffffffffu, pc, o);
                if (lane >= o) {
                    tl += a;
                    pc += b;
                }
            }
            if (e < p.n_routed) {
                s_tfirst[e] = carry_t + tl - t0;
                s_poff[e] = carry_p + pc - c;
            }
            carry_t += __shfl_sync(0xffffffffu, tl, 31);
            carry_p += __shfl_sync(0xffffffffu, pc, 31);
        }
        if (lane == 0) {
            s_tfirst[p.n_routed] = carry_t;
            s_poff[p.n_routed] = carry_p;
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;
    if (MODE == PF_ROUTER) {
        sh.n_units = ((p.E + 127) / 128) * ((p.T + kPfRouterN - 1) / kPfRouterN) * p.rchunks;
    } else {
        sh.ntiles_r = p.n_routed > 0 ? s_tfirst[p.n_routed] : 0;
        sh.pairs = p.n_routed > 0 ? s_poff[p.n_routed] : 0;
        sh.rt_r = p.side[0].rows / pf_tile_rows(MODE);
        sh.rt_s = p.side[1].rows / pf_tile_rows(MODE);
        sh.units_r = sh.ntiles_r * sh.rt_r;
        const int tiles_s = p.has_shared ? (p.T + kPfMaxN - 1) / kPfMaxN : 0;
        sh.n_units = sh.units_r + tiles_s * sh.rt_s;
    }

    if (warp == kPfProdWarp) {
        // ------------------------------------------------------------ producer
        uint32_t it_s = 0;
        bool ok = true;
        for (int u = blockIdx.x; u < sh.n_units && ok; u += gridDim.x) {
            const PfUnit un = pf_unit<MODE>(p, sh, s_tfirst, s_poff, u);
            const int N16 = (un.n + 15) & ~15;
            if (MODE == PF_ROUTER) {
                const int kst = p.H / 64, total = p.segs * kst;
                const int k0 = total * un.kc / p.rchunks, k1 = total * (un.kc + 1) / p.rchunks;
                for (int k = k0; k < k1 && ok; ++k) {
                    const int seg = k / kst, kk = (k % kst) * 64;
                    const uint32_t st = it_s & 0xFFFFu, ph = it_s >> 16;
                    int good = 1;
                    if (lane == 0) {
                        good = pf_wait_t(&empty[st], ph ^ 1u, s_abort, p.err, p.trace ? &c0 : nullptr);
                        if (good) {
                            mbar_arrive_expect_tx(&full[st], 16384u + (uint32_t)N16 * 128u);
                            tma_load_2d(smem + (size_t)st * p.stage_bytes, &p.rmap[seg == 1], kk,
                                        un.rt * 128, &full[st]);
                        }
                    }
                    ok = __shfl_sync(0xffffffffu, good, 0) != 0;
                    if (ok && 16 * lane < N16)
                        tma_load_2d(smem + (size_t)st * p.stage_bytes + p.a_bytes + 16 * lane * 128,
                                    &p.rbmap[seg == 2], kk, un.tok0 + 16 * lane,
                                    &full[st]);
                    it_s = ring_next(it_s, S);
                }
                continue;
            }
            // B: the unit's pair rows are consecutive rows of x in pair order
            // (gate/up, routed), of x (gate/up, shared) or of act (down):
            // one 128-row box and 16-row boxes per stage, kept in L2
            // (evict-last) across the row tiles of the expert
            const CUtensorMap* b128 = &p.bmap[un.side][0];
            const CUtensorMap* b16 = &p.bmap[un.side][1];
            const int row0 = (MODE == PF_GATEUP && un.side == 1) ? un.tok0 : un.prow;
            const int nb = N16 >> 7, n16 = (N16 & 127) >> 4;
            const uint64_t keep = l2_evict_last();
            const int nk = p.side[un.side].K / 64;
            for (int k = 0; k < nk && ok; ++k) {
                const uint32_t st = it_s & 0xFFFFu, ph = it_s >> 16;
                int good = 1;
                if (lane == 0) {
                    good = pf_wait_t(&empty[st], ph ^ 1u, s_abort, p.err, p.trace ? &c0 : nullptr);
                    if (good) mbar_arrive_expect_tx(&full[st], (uint32_t)N16 * 128u);
                }
                ok = __shfl_sync(0xffffffffu, good, 0) != 0;
                if (!ok) break;
                uint8_t* b = smem + (size_t)st * p.stage_bytes + p.a_bytes;
                const int k0 = 64 * k;
                if (lane < nb) {
                    tma_load_2d_hint(b + lane * 128 * 128, b128, k0, row0 + 128 * lane, &full[st],
                                     keep);
                } else if (lane < nb + n16) {
                    const int r = 128 * nb + 16 * (lane - nb);
                    tma_load_2d_hint(b + r * 128, b16, k0, row0 + r, &full[st], keep);
                }
                it_s = ring_next(it_s, S);
            }
        }
    } else if (warp == kPfRawWarp) {
        // ------------------------------------------------------ raw producer
        if (MODE != PF_ROUTER && lane == 0) {
            // the packed weights are read once per row tile: evict them first
            const uint64_t stream_pol = l2_evict_first();
            uint32_t it_r = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < sh.n_units && ok; u += gridDim.x) {
                const PfUnit un = pf_unit<MODE>(p, sh, s_tfirst, s_poff, u);
                const PfSide& sd = p.side[un.side];
                const int gv = pf_gv(sd.type), gb0 = pf_gb(sd.type), gb1 = pf_gb(sd.type2);
                const int W0 = pf_w(sd.type), W1 = pf_w(sd.type2);
                const CUtensorMap* wm0 = &p.wmap[un.side][0];
                const CUtensorMap* wm1 = &p.wmap[un.side][1];
                const int wrow = un.e * sd.rows + un.rt * pf_tile_rows(MODE);
                const uint32_t rbytes =
                    MODE == PF_GATEUP ? 64u * (uint32_t)(W0 + W1) : 128u * (uint32_t)W0;
                for (int g = 0; g < sd.K / gv; ++g) {
                    const uint32_t slot = it_r & 0xFFFFu, rph = it_r >> 16;
                    ok = pf_wait_t(&rempty[slot], rph ^ 1u, s_abort, p.err, p.trace ? &c1 : nullptr);
                    if (!ok) break;
                    uint8_t* rs = smem + (size_t)S * p.stage_bytes + (size_t)slot * p.raw_slot_bytes;
                    mbar_arrive_expect_tx(&rfull[slot], rbytes);
                    tma_load_2d_hint(rs, wm0, (g * gb0) & ~15, wrow, &rfull[slot], stream_pol);
                    if (MODE == PF_GATEUP)
                        tma_load_2d_hint(rs + 64 * W0, wm1, (g * gb1) & ~15, wrow, &rfull[slot],
                                         stream_pol);
                    it_r = ring_next(it_r, R);
                }
            }
        }
    } else if (warp == kPfMmaWarp) {
        // ------------------------------------------------------------ MMA issue
        if (lane == 0) {
            uint32_t it_s = 0, it_acc = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < sh.n_units && ok; u += gridDim.x) {
                const PfUnit un = pf_unit<MODE>(p, sh, s_tfirst, s_poff, u);
                const int N16 = (un.n + 15) & ~15;
                const uint32_t idesc = umma_idesc_f16(128, N16);
                int nk = p.side[un.side].K / 64;
                if (MODE == PF_ROUTER) {
                    const int total = p.segs * (p.H / 64);
                    nk = total * (un.kc + 1) / p.rchunks - total * un.kc / p.rchunks;
                }
                const uint32_t b = it_acc % NBUF, aph = (it_acc / NBUF) & 1u;
                ok = pf_wait_t(&acc_empty[b], aph ^ 1u, s_abort, p.err, p.trace ? &c1 : nullptr);
                if (!ok) break;
                tc_fence_after();
                const uint32_t dbase = tmem + 256u * b;
                for (int k = 0; k < nk; ++k) {
                    const uint32_t st = it_s & 0xFFFFu, ph = it_s >> 16;
                    ok = pf_wait_t(&full[st], ph, s_abort, p.err, p.trace ? &c0 : nullptr);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t a0 = smem_u32(smem + (size_t)st * p.stage_bytes);
                    const uint32_t b0 = a0 + p.a_bytes;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks)
                        umma_f16(dbase, umma_desc_sw128(a0 + 32 * ks), umma_desc_sw128(b0 + 32 * ks),
                                 idesc, (k > 0) || ks != 0);
                    umma_commit(&empty[st]);
                    it_s = ring_next(it_s, S);
                }
                if (!ok) break;
                umma_commit(&acc_full[b]);
                ++it_acc;
            }
        }
    } else if (warp < kPfEpiWarps) {
        // ------------------------------------------------------------ epilogue
        uint32_t it_acc = 0;
        const int trow = 32 * warp + lane;  // tile row = TMEM lane
        const bool tr_lane = p.trace && tid == 0;
        for (int u = blockIdx.x; u < sh.n_units; u += gridDim.x) {
            const PfUnit un = pf_unit<MODE>(p, sh, s_tfirst, s_poff, u);
            // the unit's column tokens and scales / weights, once per unit
            epi_sync();
            for (int c = tid; c < un.n; c += kPfEpiWarps * 32) {
                int tok;
                float cw;
                if (MODE == PF_ROUTER) {
                    tok = un.tok0 + c;
                    cw = p.xs_inv[tok];
                } else {
                    tok = un.side == 0 ? p.pair_tok[un.prow + c] : un.tok0 + c;
                    if (MODE == PF_GATEUP) cw = p.xs_inv[tok];
                    else cw = un.side == 0 ? p.pair_w[un.prow + c] : p.sg[tok];
                }
                s_ctok[c] = tok;
                s_cw[c] = cw;
            }
            if (epi_any(*s_abort != 0)) break;
            const uint32_t b = it_acc % NBUF, aph = (it_acc / NBUF) & 1u;
            const bool got = pf_wait_t(&acc_full[b], aph, s_abort, p.err, tr_lane ? &c0 : nullptr);
            if (epi_any(!got)) break;
            const uint64_t tb0 = tr_lane ? clock64() : 0;
            tc_fence_after();
            const uint32_t tq = tmem + ((uint32_t)(32 * warp) << 16) + 256u * b;
            for (int c0 = 0; c0 < un.n; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tq + c0, v);
                tmem_wait_ld();
                if (MODE == PF_ROUTER) {
                    // this K chunk's dot, the power-of-two scales undone (exact);
                    // the top-k kernel adds the chunks in a fixed order and the bias
                    const int e = un.rt * 128 + trow;
                    if (e < p.E) {
                        const float rs = p.rs_inv[e];
                        float* out = p.rpart + (size_t)un.kc * p.T * p.E + e;
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const int col = c0 + j;
                            if (col >= un.n) break;
                            out[(size_t)s_ctok[col] * p.E] =
                                __fmul_rn(__fmul_rn(__uint_as_float(v[j]), rs), s_cw[col]);
                        }
                    }
                } else if (MODE == PF_GATEUP) {
                    // lane pair (l, l ^ 8): gate and up of intermediate row j;
                    // the gate lane finishes even columns, the up lane odd
                    // ones.  The warp's 16 rows x 16 columns of fp16 go
                    // through shared memory so that each lane stores 16
                    // bytes (8 intermediate rows of one pair).
                    const int m = (lane >> 3) & 1;
                    const int jl = ((lane >> 4) << 3) | (lane & 7);  // 0..15 within the warp
                    __half* th = reinterpret_cast<__half*>(s_tr + warp * 256);
                    __syncwarp();
#pragma unroll
                    for (int jj = 0; jj < 16; jj += 2) {
                        const float mine0 = __uint_as_float(v[jj]);
                        const float mine1 = __uint_as_float(v[jj + 1]);
                        const float other = __shfl_xor_sync(0xffffffffu, m ? mine0 : mine1, 8);
                        const int cl = jj + m, col = c0 + cl;
                        const float g = m ? other : mine0;
                        const float uu0 = m ? mine1 : other;
                        __half ah = __float2half_rn(0.f);
                        if (col < un.n) {
                            const float xs = s_cw[col];
                            const float gg = __fmul_rn(g, xs), uu = __fmul_rn(uu0, xs);
                            // silu(g) * u with the fast exponential and divide:
                            // their ~1e-6 relative error is far below the fp16
                            // rounding of the stored activation
                            const float a = __fdividef(gg * uu, 1.0f + __expf(-gg));
                            ah = __float2half_rn(a);
                            if (!(fabsf(a) <= 65504.0f)) atomicCAS(p.err, 0u, (uint32_t)ST_RANGE);
                        }
                        th[cl * 16 + jl] = ah;
                    }
                    __syncwarp();
                    const int cl = lane >> 1, col = c0 + cl;
                    if (col < un.n) {
                        const uint4 q = *reinterpret_cast<const uint4*>(th + cl * 16 + 8 * (lane & 1));
                        *reinterpret_cast<uint4*>(p.act + (size_t)(un.prow + col) * p.Imax +
                                                  un.rt * 64 + 16 * warp + 8 * (lane & 1)) = q;
                    }
                } else {
                    // 8 columns at a time through shared memory: lane l then
                    // holds 4 consecutive hidden rows (4 (l % 8) ..) of one
                    // column and adds them with one vector reduction
                    float* tf = s_tr + warp * 256;
#pragma unroll
                    for (int half = 0; half < 2; ++half) {
                        __syncwarp();
#pragma unroll
                        for (int j = 0; j < 8; ++j) tf[j * 32 + lane] = __uint_as_float(v[8 * half + j]);
                        __syncwarp();
#pragma unroll
                        for (int it = 0; it < 2; ++it) {
                            const int cl = (lane >> 3) + 4 * it, q = lane & 7;
                            const int col = c0 + 8 * half + cl;
                            if (col < un.n) {
                                const float4 f = *reinterpret_cast<const float4*>(tf + cl * 32 + 4 * q);
                                const float wgt = s_cw[col];
                                red_add_v4(p.y + (size_t)s_ctok[col] * p.H + un.rt * 128 + 32 * warp + 4 * q,
                                           __fmul_rn(wgt, f.x), __fmul_rn(wgt, f.y),
                                           __fmul_rn(wgt, f.z), __fmul_rn(wgt, f.w));
                            }
                        }
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            ++it_acc;
            if (tr_lane) c1 += clock64() - tb0;
        }
    } else if (MODE != PF_ROUTER && warp >= kPfDqWarp0) {
        // ------------------------------------------------------------ dequant
        const int d = tid - kPfDqWarp0 * 32;
        const int h = d >> 7;
        const bool tr_on = p.trace && d == 0;
        uint32_t it_s = 0, it_r = 0;
        for (int u = blockIdx.x; u < sh.n_units; u += gridDim.x) {
            const PfUnit un = pf_unit<MODE>(p, sh, s_tfirst, s_poff, u);
            const PfSide& sd = p.side[un.side];
            int ty, trow;
            uint32_t rofs;
            if (MODE == PF_GATEUP) {
                const int m = (d >> 5) & 1;
                const int j = ((d >> 6) & 1) * 32 + lane;
                trow = ((j >> 3) << 4) | (m << 3) | (j & 7);
                ty = m ? sd.type2 : sd.type;
                rofs = m ? 64u * (uint32_t)pf_w(sd.type) + (uint32_t)(j * pf_w(sd.type2))
                         : (uint32_t)(j * pf_w(sd.type));
            } else {
                trow = d & 127;
                ty = sd.type;
                rofs = (uint32_t)(trow * pf_w(sd.type));
            }
            bool ok;
            uint64_t* t0p = tr_on ? &c0 : nullptr;
            uint64_t* t1p = tr_on ? &c1 : nullptr;
            switch (ty) {
                case Q3_K: ok = dq_unit<Q3_K, MODE>(p, un, smem, full, empty, rfull, rempty, it_s, it_r, trow, h, rofs, s_abort, t0p, t1p); break;
                case Q4_K: ok = dq_unit<Q4_K, MODE>(p, un, smem, full, empty, rfull, rempty, it_s, it_r, trow, h, rofs, s_abort, t0p, t1p); break;
                case Q5_K: ok = dq_unit<Q5_K, MODE>(p, un, smem, full, empty, rfull, rempty, it_s, it_r, trow, h, rofs, s_abort, t0p, t1p); break;
                case Q6_K: ok = dq_unit<Q6_K, MODE>(p, un, smem, full, empty, rfull, rempty, it_s, it_r, trow, h, rofs, s_abort, t0p, t1p); break;
                default:   ok = dq_unit<Q8_0, MODE>(p, un, smem, full, empty, rfull, rempty, it_s, it_r, trow, h, rofs, s_abort, t0p, t1p); break;
            }
            if (!ok) break;
        }
    }
    // --- tear-down: every MMA was waited for by the epilogue (acc_full)
    if (p.trace) {
        // slots (MODE * 10 +): 0/1 producer waits (stage empty / raw empty),
        // 2/3 dequant waits (raw full / stage empty), 4/5 MMA waits (stage
        // full / accumulator empty), 6/7 epilogue (wait / busy), 8 cycles
        // of the CTA, 9 units
        uint64_t* tr = p.trace + (size_t)blockIdx.x * 32 + MODE * 10;
        if (warp == kPfProdWarp && lane == 0) tr[0] = c0;
        if (warp == kPfRawWarp && lane == 0) tr[1] = c1;
        if (tid == kPfDqWarp0 * 32) { tr[2] = c0; tr[3] = c1; }
        if (warp == kPfMmaWarp && lane == 0) { tr[4] = c0; tr[5] = c1; }
        if (tid == 0) { tr[6] = c0; tr[7] = c1; }
    }
    tc_fence_before();
    __syncthreads();
    if (p.trace && tid == 0) {
        uint64_t* tr = p.trace + (size_t)blockIdx.x * 32 + MODE * 10;
        tr[8] = clock64() - t_start;
        int nu = 0;
        for (int u = blockIdx.x; u < sh.n_units; u += gridDim.x) ++nu;
        tr[9] = (uint64_t)nu;
    }
    if (warp == kPfMmaWarp) {
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---------------------------------------------------------------------------
// Few tokens per expert (batched decode): warp-level MMA, dequantisation
// straight into each warp's own A tile.
//
// With a handful of pairs per expert the tensor core is idle almost all the
// time and the layer's cost is the dequantisation of every weight once.
// k_bd_gemm keeps that work in the warps that consume it: a CTA of 8 warps
// owns 256 weight rows (gate/up: 128 intermediate rows, each warp 16 of
// them as 8 gate + 8 up rows per 16-row MMA tile, so that one lane holds the
// gate and the up product of the same row; down: 256 output rows) and up to
// kBdMaxN pairs; per 256-value group one thread brings the raw rows and the
// B rows (x in pair order / act, 128B-swizzled 16-row boxes) into one of two
// buffers with TMA, every lane decodes its own row of the group (the same
// functions as the tensor-core path: the exact fp16 value of the
// reference's f16 dequantisation) into the warp's 32 x 64 A tile per
// 64-value stage, and the warp runs mma.sync m16n8k16 (fp16, fp32
// accumulation) over its two row tiles and the pair tiles.  No role
// pipeline, no shared-memory handshake beyond the two group buffers.
// Epilogues as in k_pf_gemm: SiLU(g) * u to fp16 act rows, and
// y[token] += w * out with fp32 reductions.

constexpr int kBdMT = 2;                   // 16-row MMA tiles per warp
constexpr int kBdWarpRows = 16 * kBdMT;
constexpr int kBdMaxN = 64;                // pairs per unit (8 MMA column tiles)
constexpr int kBdThreads = 256;            // 8 warps
constexpr int kBdRows = 8 * kBdWarpRows;   // weight rows per unit
constexpr int kBdCtasPerSm = 1;
// Measured on the config-2 layer (Zipf-biased routing): 32 tokens 134 us per
// call on this path against 147 us on the tcgen05 pipeline, 64 tokens 168 us
// against 160 us; so up to kBdMaxT tokens take this path.
constexpr int kBdMaxT = 48;

struct BdLayout {
    uint32_t raw_bytes;   // 256 rows x W per buffer
    uint32_t buf_bytes;   // raw (rounded to 1 KB) + B tile
    uint32_t b_bytes;     // (GV / 64) stages x kBdMaxN rows x 128 B
};

__device__ __forceinline__ void bd_ldsm4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                         uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void bd_mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One unit's K loop for weight format T: buffers `bufs` (two), their
// mbarriers `bars` / phase bits `ph`; the producer thread (tid 0) issues a
// group's copies with `issue(g, buffer)`.  acc[mt][nt] accumulate the
// warp's row tile mt (16 rows) x pair tile nt (8 pairs).
// NTC: pair tiles computed (compile time; >= the unit's tiles, the columns
// past the unit's pairs are discarded by the epilogue).
template <int T, int NTC, typename Issue, typename Wait>
__device__ __forceinline__ bool bd_k_loop(int groups, uint8_t* bufs, uint32_t buf_bytes,
                                          uint32_t b_off, uint32_t raw_row_ofs, uint8_t* atile,
                                          float (&acc)[kBdMT][kBdMaxN / 8][4], Issue&& issue,
                                          Wait&& wait, volatile int* abort) {
    constexpr int GB = pf_gb(T), W = pf_w(T), NSW = W / 4, NW = PfNW<T>::n, NST = pf_gv(T) / 64;
    const int tid = threadIdx.x, lane = tid & 31;
    const uint32_t a_base = smem_u32(atile);
    for (int g = 0; g < groups; ++g) {
        const int b = g & 1;
        if (tid < 32 && g + 1 < groups) issue(g + 1, (g + 1) & 1);
        if (tid == 0) wait(b);  // group g's copies (one waiter, then the CTA)
        __syncthreads();
        if (*abort) return false;
        uint8_t* buf = bufs + (size_t)b * buf_bytes;
        // this lane's row of the group, normalised to block-relative words
        const uint8_t* rr = buf + raw_row_ofs;
        uint32_t src[NSW];
#pragma unroll
        for (int k = 0; k < W / 16; ++k) {
            const uint4 v = *reinterpret_cast<const uint4*>(rr + 16 * k);
            src[4 * k] = v.x;
            src[4 * k + 1] = v.y;
            src[4 * k + 2] = v.z;
            src[4 * k + 3] = v.w;
        }
        const int o = (g * GB) & 15;
        uint32_t w[NW];
        if (GB % 16 == 0) {
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = src[i];
        } else {
            const int q = o >> 2;
            const uint32_t sb = (uint32_t)(o & 3) * 8u;
            uint32_t t1[NSW];
#pragma unroll
            for (int i = 0; i < NSW; ++i) t1[i] = (q & 1) ? (i + 1 < NSW ? src[i + 1] : 0u) : src[i];
#pragma unroll
            for (int i = 0; i < NSW; ++i) src[i] = (q & 2) ? (i + 2 < NSW ? t1[i + 2] : 0u) : t1[i];
#pragma unroll
            for (int i = 0; i < NW; ++i) w[i] = __funnelshift_r(src[i], src[i + 1], sb);
        }
        const uint32_t b_base0 = smem_u32(buf + b_off);
        auto stage = [&](auto s_c) {
            constexpr int S = decltype(s_c)::value;
            if constexpr (kBdMT == 2) {
                dq_store<T, S>(atile, lane, 0, w);
                dq_store<T, S>(atile, lane, 1, w);
            } else {
                dq_store<T, S>(atile, lane & 15, lane >> 4, w);  // two lanes per row
            }
            __syncwarp();
            const uint32_t b_base = b_base0 + (uint32_t)(S * kBdMaxN * 128);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t a[kBdMT][4];
#pragma unroll
                for (int mt = 0; mt < kBdMT; ++mt) {
                    const int r = 16 * mt + (lane & 7) + 8 * ((lane >> 3) & 1), c = 2 * ks + (lane >> 4);
                    bd_ldsm4(a_base + sw128_offset(r, c), a[mt][0], a[mt][1], a[mt][2], a[mt][3]);
                }
#pragma unroll
                for (int nt = 0; nt < NTC; nt += 2) {
                    const int n = 8 * nt + (lane & 7) + 8 * (lane >> 4), c = 2 * ks + ((lane >> 3) & 1);
                    uint32_t b0, b1, b2, b3;
                    bd_ldsm4(b_base + sw128_offset(n, c), b0, b1, b2, b3);
#pragma unroll
                    for (int mt = 0; mt < kBdMT; ++mt) {
                        bd_mma(acc[mt][nt], a[mt], b0, b1);
                        bd_mma(acc[mt][nt + 1], a[mt], b2, b3);
                    }
                }
            }
            __syncwarp();
        };
        stage(std::integral_constant<int, 0>{});
        stage(std::integral_constant<int, 1>{});
        if constexpr (NST == 4) {
            stage(std::integral_constant<int, 2>{});
            stage(std::integral_constant<int, 3>{});
        }
        __syncthreads();  // buffer b free for group g + 2
    }
    return true;
}

template <int MODE>
__global__ void __launch_bounds__(kBdThreads, kBdCtasPerSm) k_bd_gemm(const __grid_constant__ PfParams p) {
    pdl_enter();
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    // layout: two group buffers, 8 warp A tiles (32 rows x 128 B), control
    uint8_t* bufs = smem;
    const uint32_t buf_bytes = p.stage_bytes;  // per buffer (raw rows + B tile)
    uint8_t* atiles = smem + 2 * (size_t)buf_bytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(atiles + 8 * kBdWarpRows * 128);
    volatile int* s_abort = reinterpret_cast<volatile int*>(bars + 2);
    int* s_tfirst = reinterpret_cast<int*>(bars + 3);
    int* s_poff = s_tfirst + (p.n_routed + 1);
    uint8_t* atile = atiles + warp * kBdWarpRows * 128;

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        *s_abort = 0;
        mbar_fence_init();
    }
    if (warp == 0) {
        // column tiles and pair offsets of the held experts (exclusive prefix sums)
        int carry_t = 0, carry_p = 0;
        for (int base = 0; base < p.n_routed; base += 32) {
            const int e = base + lane;
            const int c = e < p.n_routed ? p.counts[e] : 0;
            const int t0 = (c + kBdMaxN - 1) / kBdMaxN;
            int tl = t0, pc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int a = __shfl_up_sync(0xffffffffu, tl, o);
                const int b = __shfl_up_sync(0xffffffffu, pc, o);
                if (lane >= o) {
                    tl += a;
                    pc += b;
                }
            }
            if (e < p.n_routed) {
                s_tfirst[e] = carry_t + tl - t0;
                s_poff[e] = carry_p + pc - c;
            }
            carry_t += __shfl_sync(0xffffffffu, tl, 31);
            carry_p += __shfl_sync(0xffffffffu, pc, 31);
        }
        if (lane == 0) {
            s_tfirst[p.n_routed] = carry_t;
            s_poff[p.n_routed] = carry_p;
        }
    }
    __syncthreads();
    constexpr int RPU = MODE == PF_GATEUP ? kBdRows / 2 : kBdRows;  // side rows per unit
    const int ntiles_r = p.n_routed > 0 ? s_tfirst[p.n_routed] : 0;
    const int pairs = p.n_routed > 0 ? s_poff[p.n_routed] : 0;
    const int rt_r = p.side[0].rows / RPU, rt_s = p.side[1].rows / RPU;
    const int units_r = ntiles_r * rt_r;
    const int tiles_s = p.has_shared ? (p.T + kBdMaxN - 1) / kBdMaxN : 0;
    const int n_units = units_r + tiles_s * rt_s;
    const uint64_t stream_pol = l2_evict_first(), keep = l2_evict_last();
    uint32_t ph = 0, pend = 0;  // (thread 0) phase bit and copies in flight, per buffer
    auto wait = [&](int b) {     // thread 0: bounded wait for buffer b's copies
        bool okw = false;
        for (uint32_t i = 0; i < kPfPolls; ++i)
            if (mbar_try_wait(&bars[b], (ph >> b) & 1u)) {
                okw = true;
                break;
            }
        ph ^= 1u << b;
        pend &= ~(1u << b);
        if (!okw) {
            atomicCAS(p.err, 0u, (uint32_t)ST_TIMEOUT);
            *s_abort = 1;
        }
    };
    constexpr int kBoxRows = MODE == PF_GATEUP ? 64 : 128;  // rows of a raw weight box

    // units are taken from a work counter (workspace word 16 + MODE), the
    // shared expert's first: they have a column per token, the heaviest
    uint32_t* work = p.err + 8 + 2 * MODE;  // [0] next unit, [1] CTAs done
    int* s_unit = s_poff + (p.n_routed + 1);
    const int units_s = n_units - units_r;
    for (;;) {
        if (tid == 0) *s_unit = (int)atomicAdd(work, 1u);
        __syncthreads();
        const int uw = *s_unit;
        __syncthreads();
        if (uw >= n_units) break;
        const int u = uw < units_s ? units_r + uw : uw - units_s;
        // ---- the unit: side, expert, row tile, pairs
        int side, e = 0, rt, n, prow, tok0 = 0;
        if (u < units_r) {
            const int tile = u / rt_r;
            side = 0;
            rt = u % rt_r;
            int lo = 0, hi = p.n_routed;
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (s_tfirst[mid] <= tile) lo = mid;
                else hi = mid;
            }
            e = lo;
            prow = s_poff[e] + (tile - s_tfirst[e]) * kBdMaxN;
            n = min(kBdMaxN, s_poff[e + 1] - prow);
        } else {
            const int v = u - units_r;
            side = 1;
            rt = v % rt_s;
            tok0 = (v / rt_s) * kBdMaxN;
            n = min(kBdMaxN, p.T - tok0);
            prow = pairs + tok0;
        }
        const PfSide& sd = p.side[side];
        const int W0 = pf_w(sd.type), W1 = pf_w(sd.type2), GV = pf_gv(sd.type);
        const int GB0 = pf_gb(sd.type), GB1 = pf_gb(sd.type2);
        const int groups = sd.K / GV, nst = GV / 64;
        const int N16 = (n + 15) & ~15, ntv = (n + 7) / 8;
        const int wrow = e * sd.rows + rt * RPU;   // first weight row of the unit (per matrix)
        const int brow = (MODE == PF_GATEUP && side == 1) ? tok0 : prow;   // first B row
        const uint32_t raw_bytes = MODE == PF_GATEUP ? (uint32_t)(RPU * (W0 + W1)) : (uint32_t)(RPU * W0);
        const uint32_t b_off = (raw_bytes + 1023u) & ~1023u;
        // a group's copies, issued by the lanes of warp 0 together: lanes
        // 0..nraw-1 one raw box each, the next lanes one 16-row B box each
        // (lane 0 posts the byte count first)
        const int nraw = (MODE == PF_GATEUP ? 2 : 1) * (RPU / kBoxRows);
        const int nb16 = N16 / 16;
        auto issue = [&](int g, int b) {
            uint8_t* buf = bufs + (size_t)b * buf_bytes;
            if (lane == 0) {
                pend |= 1u << b;
                mbar_arrive_expect_tx(&bars[b], raw_bytes + (uint32_t)(nst * N16 * 128));
            }
            __syncwarp();
            if (lane < nraw) {
                const int m = lane / (RPU / kBoxRows), q = lane % (RPU / kBoxRows);
                if (m == 0)
                    tma_load_2d_hint(buf + q * kBoxRows * W0, &p.wmap[side][0], (g * GB0) & ~15,
                                     wrow + kBoxRows * q, &bars[b], stream_pol);
                else
                    tma_load_2d_hint(buf + RPU * W0 + q * kBoxRows * W1, &p.wmap[side][1],
                                     (g * GB1) & ~15, wrow + kBoxRows * q, &bars[b], stream_pol);
            }
            for (int i = lane - nraw; i >= 0 && i < nst * nb16; i += 32 - nraw) {
                const int st = i / nb16, r = 16 * (i % nb16);
                tma_load_2d_hint(buf + b_off + (uint32_t)(st * kBdMaxN * 128) + r * 128, &p.bmap[side][1],
                                 g * GV + 64 * st, brow + r, &bars[b], keep);
            }
        };
        if (warp == 0) issue(0, 0);
        // ---- this lane's weight row: 16-row MMA tiles mt = lane / 16
        uint32_t rofs;
        int ty;
        // (two m-tiles: lane = staging row; one m-tile: lanes l and l + 16
        // share staging row l % 16)
        const int srow = kBdMT == 2 ? lane : (lane & 15);
        if (MODE == PF_GATEUP) {
            const int mt = srow >> 4, rr = srow & 15;
            const int j = kBdWarpRows / 2 * warp + 8 * mt + (rr & 7);   // intermediate row in the unit
            const bool up = rr >= 8;
            rofs = up ? (uint32_t)(RPU * W0 + j * W1) : (uint32_t)(j * W0);
            ty = up ? sd.type2 : sd.type;
        } else {
            rofs = (uint32_t)((kBdWarpRows * warp + srow) * W0);
            ty = sd.type;
        }
        float acc[kBdMT][kBdMaxN / 8][4];
#pragma unroll
        for (int mt = 0; mt < kBdMT; ++mt)
#pragma unroll
            for (int nt = 0; nt < kBdMaxN / 8; ++nt)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[mt][nt][j] = 0.f;
        // one decoder and a pair-tile count known at compile time per unit
        auto run = [&](auto t_c) -> bool {
            constexpr int TT = decltype(t_c)::value;
            if (ntv <= 2) return bd_k_loop<TT, 2>(groups, bufs, buf_bytes, b_off, rofs, atile, acc, issue, wait, s_abort);
            if (kBdMaxN <= 32 || ntv <= 4) return bd_k_loop<TT, (kBdMaxN <= 32 ? kBdMaxN / 8 : 4)>(groups, bufs, buf_bytes, b_off, rofs, atile, acc, issue, wait, s_abort);
            return bd_k_loop<TT, kBdMaxN / 8>(groups, bufs, buf_bytes, b_off, rofs, atile, acc, issue, wait, s_abort);
        };
        bool ok;
        switch (ty) {
            case Q3_K: ok = run(std::integral_constant<int, Q3_K>{}); break;
            case Q4_K: ok = run(std::integral_constant<int, Q4_K>{}); break;
            case Q5_K: ok = run(std::integral_constant<int, Q5_K>{}); break;
            case Q6_K: ok = run(std::integral_constant<int, Q6_K>{}); break;
            default:   ok = run(std::integral_constant<int, Q8_0>{}); break;
        }
        if (!ok) break;
        __syncthreads();  // the next unit's first copies reuse buffer 0
        // ---- epilogue: C fragment rows g (c0, c1) and g + 8 (c2, c3), columns 2t, 2t + 1
        const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
        for (int nt = 0; nt < kBdMaxN / 8; ++nt) {
            if (nt >= ntv) break;
#pragma unroll
            for (int ec = 0; ec < 2; ++ec) {
                const int col = 8 * nt + 2 * tq + ec;
                if (col >= n) continue;
                int tok;
                if (side == 0) tok = p.pair_tok[prow + col];
                else tok = tok0 + col;
#pragma unroll
                for (int mt = 0; mt < kBdMT; ++mt) {
                    if (MODE == PF_GATEUP) {
                        // row gq of tile mt is gate row j, row gq + 8 the up row j
                        const int j = rt * RPU + kBdWarpRows / 2 * warp + 8 * mt + gq;
                        const float xs = p.xs_inv[tok];
                        const float gg = __fmul_rn(acc[mt][nt][ec], xs);
                        const float uu = __fmul_rn(acc[mt][nt][2 + ec], xs);
                        const float a = __fdividef(gg * uu, 1.0f + __expf(-gg));
                        if (!(fabsf(a) <= 65504.0f)) atomicCAS(p.err, 0u, (uint32_t)ST_RANGE);
                        p.act[(size_t)(prow + col) * p.Imax + j] = __float2half_rn(a);
                    } else {
                        const float wgt = side == 0 ? p.pair_w[prow + col] : p.sg[tok];
                        const int h = rt * RPU + kBdWarpRows * warp + 16 * mt + gq;
                        float* yr = p.y + (size_t)tok * p.H;
                        atomicAdd(yr + h, __fmul_rn(wgt, acc[mt][nt][ec]));
                        atomicAdd(yr + h + 8, __fmul_rn(wgt, acc[mt][nt][2 + ec]));
                    }
                }
            }
        }
    }
    // after an abort: let the copies still in flight land before the CTA's
    // shared memory goes away (bounded)
    if (tid == 0)
        for (int b = 0; b < 2; ++b)
            if (pend & (1u << b))
                for (uint32_t i = 0; i < kPfPolls; ++i)
                    if (mbar_try_wait(&bars[b], (ph >> b) & 1u)) break;
    // the last CTA out resets the work counter for the next call
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(work + 1, 1u) == gridDim.x - 1) {
            work[0] = 0;
            work[1] = 0;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------
// token and router preparation, top-k, pair lists

struct PfPrep {
    int T, H, E, n_routed, x_bf16;
    int want_lo;            // write xl (the tensor-core router's lo half of x)
    const void* x;
    const float* gate_inp;  // [H] or null
    const float* router;    // [E x H]
    __half* xh;
    __half* xl;
    __half* rh;
    __half* rl;
    float* xs_inv;
    float* rs_inv;
    float* sg;
    float* y;
    int32_t* counts;
    int32_t* cursor;
};

__device__ __forceinline__ float pf_x(const PfPrep& p, size_t i) {
    return p.x_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.x)[i])
                    : reinterpret_cast<const float*>(p.x)[i];
}

// Power of two 2^k with amax * 2^k in [2^14, 2^15) (k clamped to +-126).
__device__ __forceinline__ int pf_scale_exp(float amax) {
    if (!(amax > 0.f) || !isfinite(amax)) return 0;
    int e;
    frexpf(amax, &e);  // amax in [2^(e-1), 2^e)
    return max(-126, min(126, 15 - e));
}

// Eight consecutive values of x (fp32 or bf16) from element i (a multiple of
// 8); `vec`: x is 16-byte aligned, so one or two 16-byte loads do.
__device__ __forceinline__ void pf_x8(const PfPrep& p, size_t i, bool vec, float (&v)[8]) {
    if (vec && p.x_bf16) {
        const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.x) + i);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            v[2 * q] = __uint_as_float(w[q] << 16);
            v[2 * q + 1] = __uint_as_float(w[q] & 0xFFFF0000u);
        }
    } else if (vec) {
        const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + i);
        const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + i + 4);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = pf_x(p, i + q);
    }
}

// Chunks of 8 values a thread of k_pf_prep_x holds in registers: the row is
// read once (H <= 256 * 8 * kPfPrepChunks).
constexpr int kPfPrepChunks = 4;

// one block (256 threads) per token; block 0 also clears the pair counts and
// the pair cursors of the held experts
__global__ void __launch_bounds__(256) k_pf_prep_x(PfPrep p) {
    pdl_enter();
    __shared__ float s_red[2][8];
    const int t = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (t == 0)
        for (int i = tid; i < p.n_routed; i += blockDim.x) {
            p.counts[i] = 0;
            p.cursor[i] = 0;
        }
    const size_t base = (size_t)t * p.H;
    const int nch = p.H / 8;
    const bool vx = ((uintptr_t)p.x & 15u) == 0;
    const bool vg = p.gate_inp && ((uintptr_t)p.gate_inp & 15u) == 0;
    const bool vy = ((uintptr_t)p.y & 15u) == 0;
    float v[kPfPrepChunks][8];
    float amax = 0.f, dot = 0.f;
#pragma unroll
    for (int j = 0; j < kPfPrepChunks; ++j) {
        const int c = tid + 256 * j;
        if (c >= nch) break;
        pf_x8(p, base + 8 * (size_t)c, vx, v[j]);
#pragma unroll
        for (int q = 0; q < 8; ++q) amax = fmaxf(amax, fabsf(v[j][q]));
        if (p.gate_inp) {
            float g[8];
            if (vg) {
                const float4 a = *reinterpret_cast<const float4*>(p.gate_inp + 8 * c);
                const float4 b = *reinterpret_cast<const float4*>(p.gate_inp + 8 * c + 4);
                g[0] = a.x; g[1] = a.y; g[2] = a.z; g[3] = a.w;
                g[4] = b.x; g[5] = b.y; g[6] = b.z; g[7] = b.w;
            } else {
#pragma unroll
                for (int q = 0; q < 8; ++q) g[q] = p.gate_inp[8 * c + q];
            }
#pragma unroll
            for (int q = 0; q < 8; ++q) dot = fmaf(v[j][q], g[q], dot);
        }
        float* yr = p.y + base + 8 * (size_t)c;
        if (vy) {
            reinterpret_cast<float4*>(yr)[0] = make_float4(0.f, 0.f, 0.f, 0.f);
            reinterpret_cast<float4*>(yr)[1] = make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
#pragma unroll
            for (int q = 0; q < 8; ++q) yr[q] = 0.f;
        }
    }
    amax = warp_max(amax);
    if (p.gate_inp) dot = warp_sum(dot);
    if (lane == 0) {
        s_red[0][warp] = amax;
        s_red[1][warp] = dot;
    }
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, s_red[0][i]);
    const int k = pf_scale_exp(amax);
    const float sc = ldexpf(1.f, k);
#pragma unroll
    for (int j = 0; j < kPfPrepChunks; ++j) {
        const int c = tid + 256 * j;
        if (c >= nch) break;
        uint32_t hw[4], lw[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float a = __fmul_rn(v[j][2 * q], sc), b = __fmul_rn(v[j][2 * q + 1], sc);
            const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
            hw[q] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
            const __half la = __float2half_rn(__fsub_rn(a, __half2float(ha)));
            const __half lb = __float2half_rn(__fsub_rn(b, __half2float(hb)));
            lw[q] = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
        }
        *reinterpret_cast<uint4*>(p.xh + base + 8 * (size_t)c) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        if (p.want_lo)
            *reinterpret_cast<uint4*>(p.xl + base + 8 * (size_t)c) = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    }
    if (tid == 0) {
        p.xs_inv[t] = ldexpf(1.f, -k);
        if (p.gate_inp) {
            // the shared-gate dot in a fixed order: warps 0..7
            float d = 0.f;
            for (int i = 0; i < 8; ++i) d += s_red[1][i];
            p.sg[t] = shared_sigmoid(d);
        }
    }
}

struct PfRoute {
    int T, E, K, expert_begin, n_routed;
    float* logits;
    const float* part;     // null, or [nparts x T x E] scaled partial logits of the
    int nparts;            // tensor-core router, added here in a fixed order
    const float* bias;     // with part: the router bias [E] or null
    int32_t* ids;
    float* w;
    int32_t* ids_out;
    float* w_out;
    int32_t* counts;
    int32_t* cursor;       // [n_routed] slots taken per held expert (zero on entry)
    int32_t* pair_tok;
    float* pair_w;
};

// After a token's selection (ids, w of token t): the caller's routing rows
// and the pair count of each held expert (lanes 0..K-1).
__device__ __forceinline__ void pf_route_emit(const PfRoute& p, int t, const int32_t* ids,
                                              const float* w, int lane) {
    __syncwarp();
    if (lane < p.K) {
        const int id = ids[lane];
        if (p.ids_out) p.ids_out[(size_t)t * p.K + lane] = id;
        if (p.w_out) p.w_out[(size_t)t * p.K + lane] = w[lane];
        const int local = id - p.expert_begin;
        if (local >= 0 && local < p.n_routed) atomicAdd(&p.counts[local], 1);
    }
}

// Token t's logits from the tensor-core router's K-chunk partials: added
// in a fixed order (eight: ((p0 + p1) + (p2 + p3)) + ((p4 + p5) + (p6 + p7)),
// else in chunk order), then the bias.  One warp; the sums go to p.logits.
__device__ __forceinline__ void pf_logits_from_parts(const PfRoute& p, int t, int lane) {
    const size_t stride = (size_t)p.T * p.E;
    for (int e = lane; e < p.E; e += 32) {
        const float* q = p.part + (size_t)t * p.E + e;
        float v;
        if (p.nparts == 8) {
            float a[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) a[j] = __ldcg(q + j * stride);
            v = __fadd_rn(__fadd_rn(__fadd_rn(a[0], a[1]), __fadd_rn(a[2], a[3])),
                          __fadd_rn(__fadd_rn(a[4], a[5]), __fadd_rn(a[6], a[7])));
        } else {
            v = __ldcg(q);
            for (int j = 1; j < p.nparts; ++j) v = __fadd_rn(v, __ldcg(q + j * stride));
        }
        if (p.bias) v = __fadd_rn(v, p.bias[e]);
        p.logits[(size_t)t * p.E + e] = v;
    }
    __syncwarp();
}

// Top-k and weights of token t for E <= 256 (one warp, scores through L2).
__device__ __forceinline__ void pf_route_token(const PfRoute& p, int t, int lane) {
    int32_t* ids = p.ids + (size_t)t * p.K;
    float* w = p.w + (size_t)t * p.K;
    topk_softmax_warp_fast(p.logits + (size_t)t * p.E, p.E, p.K, ids, w);
    pf_route_emit(p, t, ids, w, lane);
}

// Router logits of a few tokens on the CUDA cores, in fp32, for T <=
// kPfSmallRouterT (where the tensor-core router would run on a handful of
// SMs).  Block (x, y) computes the kRsE x kRsTok dots of experts
// [kRsE x, +kRsE) with tokens [kRsTok y, +kRsTok): thread i sums the hidden
// quads i, i + 256, ... (all its loads in flight at once), a warp folds its
// 32 lanes' partial sums with a butterfly reduce-scatter, and the 8 warps'
// sums are added in warp order (a fixed order: deterministic); then the
// bias.  Needs 16-byte aligned router rows and tokens.
constexpr int kPfSmallRouterT = 128;
constexpr int kRsE = 8, kRsTok = 8;

__device__ __forceinline__ float4 pf_x4(const PfPrep& p, size_t i) {  // i a multiple of 4
    if (p.x_bf16) {
        const uint2 v = *reinterpret_cast<const uint2*>(reinterpret_cast<const __nv_bfloat16*>(p.x) + i);
        return make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
    }
    return *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.x) + i);
}

// With `tcnt` (an arrival counter per token tile, zero between calls; E <=
// 256) the last block of a token tile to finish also routes its tokens, one
// warp per token: the top-k kernel's work without its launch.
__global__ void __launch_bounds__(256) k_pf_router_small(PfPrep p, const float* bias,
                                                         float* logits, PfRoute rp,
                                                         uint32_t* tcnt) {
    pdl_enter();
    __shared__ float s_part[8][kRsE * kRsTok];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int e0 = blockIdx.x * kRsE, t0 = blockIdx.y * kRsTok;
    const int ne = min(kRsE, p.E - e0), nt = min(kRsTok, p.T - t0);
    float acc[kRsE * kRsTok];
#pragma unroll
    for (int i = 0; i < kRsE * kRsTok; ++i) acc[i] = 0.f;
    for (int q = tid; q < p.H / 4; q += 256) {
        float4 rv[kRsE], xv[kRsTok];
#pragma unroll
        for (int e = 0; e < kRsE; ++e)
            rv[e] = e < ne ? *reinterpret_cast<const float4*>(p.router + (size_t)(e0 + e) * p.H + 4 * q)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int t = 0; t < kRsTok; ++t)
            xv[t] = t < nt ? pf_x4(p, (size_t)(t0 + t) * p.H + 4 * q) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int e = 0; e < kRsE; ++e) {
#pragma unroll
            for (int t = 0; t < kRsTok; ++t) {
                float a = acc[e * kRsTok + t];
                a = fmaf(rv[e].x, xv[t].x, a);
                a = fmaf(rv[e].y, xv[t].y, a);
                a = fmaf(rv[e].z, xv[t].z, a);
                a = fmaf(rv[e].w, xv[t].w, a);
                acc[e * kRsTok + t] = a;
            }
        }
    }
    // reduce-scatter over the warp: after the step with offset o a lane keeps
    // the half of its values selected by its bit o; lane l ends with the sums
    // of values 2l and 2l + 1
#pragma unroll
    for (int o = 16, n = kRsE * kRsTok; o >= 1; o >>= 1, n >>= 1) {
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i) {
            const float send = up ? acc[i] : acc[i + n / 2];
            const float keep = up ? acc[i + n / 2] : acc[i];
            acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
    }
    s_part[warp][2 * lane] = acc[0];
    s_part[warp][2 * lane + 1] = acc[1];
    __syncthreads();
    if (tid < kRsE * kRsTok) {
        const int e = tid / kRsTok, t = tid % kRsTok;
        if (e < ne && t < nt) {
            float v = 0.f;
            for (int w = 0; w < 8; ++w) v += s_part[w][tid];
            if (bias) v = __fadd_rn(v, bias[e0 + e]);
            logits[(size_t)(t0 + t) * p.E + e0 + e] = v;
        }
    }
    if (!tcnt) return;
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(tcnt + blockIdx.y, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (warp < nt) pf_route_token(rp, t0 + warp, lane);
    if (tid == 0) tcnt[blockIdx.y] = 0;  // ready for the next call
}

// one block per router row
__global__ void __launch_bounds__(256) k_pf_prep_router(PfPrep p) {
    pdl_enter();
    __shared__ float s_red[8];
    const int e = blockIdx.x;
    const float* r = p.router + (size_t)e * p.H;
    float amax = 0.f;
    for (int i = threadIdx.x; i < p.H; i += blockDim.x) amax = fmaxf(amax, fabsf(r[i]));
    amax = warp_max(amax);
    if ((threadIdx.x & 31) == 0) s_red[threadIdx.x >> 5] = amax;
    __syncthreads();
    amax = 0.f;
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, s_red[i]);
    const int k = pf_scale_exp(amax);
    const float sc = ldexpf(1.f, k);
    for (int i = threadIdx.x; i < p.H; i += blockDim.x) {
        const float v = __fmul_rn(r[i], sc);
        const __half hi = __float2half_rn(v);
        p.rh[(size_t)e * p.H + i] = hi;
        p.rl[(size_t)e * p.H + i] = __float2half_rn(__fsub_rn(v, __half2float(hi)));
    }
    if (threadIdx.x == 0) p.rs_inv[e] = ldexpf(1.f, -k);
}


// one warp per token, up to kPfTopkWarps tokens per block (blocks of one
// warp spent more time being scheduled than routing)
constexpr int kPfTopkWarps = 8;
__global__ void __launch_bounds__(32 * kPfTopkWarps) k_pf_topk(PfRoute p) {
    pdl_enter();
    extern __shared__ float s_sc[];
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (t >= p.T) return;
    if (p.part) pf_logits_from_parts(p, t, lane);
    if (p.E <= 256) {
        pf_route_token(p, t, lane);
        return;
    }
    int32_t* ids = p.ids + (size_t)t * p.K;
    float* w = p.w + (size_t)t * p.K;
    // this warp's scores and taken flags: E floats + E bytes, 16-byte aligned
    float* sc = s_sc + (size_t)(threadIdx.x >> 5) * (((size_t)p.E * 5 + 15) / 16 * 4);
    unsigned char* taken = reinterpret_cast<unsigned char*>(sc + p.E);
    for (int e = lane; e < p.E; e += 32) sc[e] = p.logits[(size_t)t * p.E + e];
    __syncwarp();
    topk_softmax_warp(sc, taken, p.E, p.K, ids, w);
    pf_route_emit(p, t, ids, w, lane);
}

// One warp per (token, slot) pair: a pair of a held expert takes the next
// place of that expert's list -- the expert's offset (the exclusive prefix
// sum of the pair counts, which every block forms itself) plus a slot from
// the expert's cursor -- and the warp copies the token's fp16 row there (the
// gate/up GEMM's B rows, an expert's pairs contiguous).  The order within an
// expert's list is the order the slots were taken; each pair's GEMM result
// does not depend on its column.
__global__ void __launch_bounds__(256) k_pf_pairs(PfRoute p, const __half* xh, __half* xperm,
                                                  int H) {
    pdl_enter();
    __shared__ int s_off[kPfMaxExperts];
    __shared__ int s_w[8];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int carry = 0;
    for (int base = 0; base < p.n_routed; base += 256) {
        const int e = base + tid;
        const int c = e < p.n_routed ? p.counts[e] : 0;
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        if (lane == 31) s_w[warp] = incl;
        __syncthreads();
        int before = 0, total = 0;
        for (int i = 0; i < 8; ++i) {
            if (i < warp) before += s_w[i];
            total += s_w[i];
        }
        if (e < p.n_routed) s_off[e] = carry + before + incl - c;
        carry += total;
        __syncthreads();
    }
    if (blockIdx.x == 0 && tid == 0) p.counts[p.n_routed] = carry;  // pairs in total
    const int i = blockIdx.x * 8 + warp;
    if (i >= p.T * p.K) return;
    const int local = p.ids[i] - p.expert_begin;
    if (local < 0 || local >= p.n_routed) return;
    int pos = 0;
    if (lane == 0) pos = s_off[local] + atomicAdd(&p.cursor[local], 1);
    pos = __shfl_sync(0xffffffffu, pos, 0);
    const int t = i / p.K;
    if (lane == 0) {
        p.pair_tok[pos] = t;
        p.pair_w[pos] = p.w[i];
    }
    const uint4* src = reinterpret_cast<const uint4*>(xh + (size_t)t * H);
    uint4* dst = reinterpret_cast<uint4*>(xperm + (size_t)pos * H);
    for (int j = lane; j < H / 8; j += 32) dst[j] = src[j];
}

// ---------------------------------------------------------------------------
// host side

// Calls of at most this many tokens launch their kernels with programmatic
// stream serialization: each prefill kernel begins with pdl_enter, so it may
// start launching while the previous kernel of the stream finishes, which
// hides most of the gap between a small call's short kernels (B200: 32
// tokens 123 -> 114 us, 64 tokens 135 -> 130 us per call).  A 4096-token
// call was slower that way (671 -> 697 us) and launches plainly.
constexpr int kPfPdlMaxT = kPfSmallRouterT;

template <typename... P, typename... A>
static cudaError_t pf_launch(int T, void (*k)(P...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t s, A&&... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    // MOE_B200_NO_PDL (diagnostics): plain launches, so that a profiler's
    // kernel spans do not include the programmatic wait for the previous one
    cfg.numAttrs = (T <= kPfPdlMaxT && !std::getenv("MOE_B200_NO_PDL")) ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k, std::forward<A>(args)...);
}

static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    return fn;
}

// 2-D map over a row-major matrix: inner extent `cols` elements, `rows`
// rows, row pitch `pitch` bytes, box {bx, by}.
static bool make_map(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t cols,
                     uint64_t rows, uint64_t pitch, uint32_t bx, uint32_t by, bool swz) {
    auto enc = tmap_encoder();
    if (!enc) return false;
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {pitch};
    cuuint32_t box[2] = {bx, by};
    cuuint32_t es[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE,
               swz ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) ==
           CUDA_SUCCESS;
}

static bool pf_type_ok(int t) {
    return t == Q8_0 || t == Q3_K || t == Q4_K || t == Q5_K || t == Q6_K;
}

bool prefill_supported(const moe_b200_layer* L, int flags) {
    if (flags & (MOE_B200_EXACT | MOE_B200_FP16_GRAPH)) return false;
    const bool routed = !(flags & MOE_B200_SHARED_ONLY);
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    if (!routed && !shared) return false;
    if (L->hidden % 256 || L->hidden <= 0 || L->hidden > 256 * 8 * kPfPrepChunks) return false;
    if (routed) {
        if (L->expert_count <= 0 || L->expert_count > kPfMaxExperts) return false;
        if (L->top_k < 1 || L->top_k > kMaxTopK || L->n_experts > 4096) return false;
        if (L->intermediate % 256 || L->intermediate <= 0) return false;
        const int ty[3] = {L->gate_type, L->up_type, L->down_type};
        const int cols[3] = {L->hidden, L->hidden, L->intermediate};
        for (int i = 0; i < 3; ++i)
            if (!pf_type_ok(ty[i]) || row_bytes(ty[i], cols[i]) % 16) return false;
        if (pf_gv(L->gate_type) != pf_gv(L->up_type)) return false;
    }
    if (shared) {
        if (L->shared_intermediate % 256) return false;
        const int ty[3] = {L->shared_gate_type, L->shared_up_type, L->shared_down_type};
        const int cols[3] = {L->hidden, L->hidden, L->shared_intermediate};
        for (int i = 0; i < 3; ++i)
            if (!pf_type_ok(ty[i]) || row_bytes(ty[i], cols[i]) % 16) return false;
        if (pf_gv(L->shared_gate_type) != pf_gv(L->shared_up_type)) return false;
    }
    return true;
}

struct PfWs {
    size_t counts, cursor, xs_inv, sg, xh, xl, rh, rl, rs_inv, logits, rpart, ids, w, ptok, pw, act, xperm,
        total;
};

// The CUDA-core router for few tokens (needs 16-byte aligned router rows).
// Its per-token-tile arrival counters (at most 32 tiles of kRsTok tokens)
// live in bytes [128, 256) of the workspace, among the control words that
// stay zero between calls.
constexpr int kRsCntOffset = 128;
static_assert(kPfSmallRouterT / kRsTok <= (256 - kRsCntOffset) / 4, "token tiles");
static bool pf_small_router(const moe_b200_layer* L, int T) {
    return T <= kPfSmallRouterT && ((uintptr_t)L->router & 15u) == 0;
}

static PfWs pf_ws(const moe_b200_layer* L, int T) {
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate
                                                              : L->intermediate;
    const size_t H = L->hidden, E = L->n_experts, K = L->top_k;
    Stager s;
    s.used = 256;
    PfWs w;
    w.counts = s.take((size_t)(L->expert_count + 1) * 4);
    w.cursor = s.take((size_t)L->expert_count * 4);
    w.xs_inv = s.take((size_t)T * 4);
    w.sg = s.take((size_t)T * 4);
    w.xh = s.take((size_t)T * H * 2);
    w.xl = s.take((size_t)T * H * 2);
    w.rh = s.take(E * H * 2);
    w.rl = s.take(E * H * 2);
    w.rs_inv = s.take(E * 4);
    w.logits = s.take((size_t)T * E * 4);
    w.rpart = s.take((size_t)kPfRouterChunks * T * E * 4);
    w.ids = s.take((size_t)T * K * 4);
    w.w = s.take((size_t)T * K * 4);
    w.ptok = s.take((size_t)T * K * 4);
    w.pw = s.take((size_t)T * K * 4);
    w.act = s.take(((size_t)T * K + T) * Imax * 2);
    w.xperm = s.take((size_t)T * K * H * 2);
    w.total = s.used;
    return w;
}

size_t prefill_workspace_bytes(const moe_b200_layer* L, int T) { return pf_ws(L, T).total; }

// shared memory after the stages and raw slots: mbarriers, TMEM address,
// abort flag, the epilogue's column tokens and scales, the tile prefixes
static size_t pf_ctrl_bytes(const PfParams& p) {
    return (size_t)(2 * p.stages + 2 * p.raw_slots + 4) * 8 + 16 + (size_t)2 * kPfMaxN * 4 +
           (size_t)4 * 256 * 4 + (size_t)2 * (p.n_routed + 1) * 4;
}

// Stages (up to 6) and raw slots (up to 4) that fit the shared memory: the
// most stages that leave room for three raw slots, else two stages.  Few
// tokens make small stages (the B rows of a stage are the unit's columns),
// so small calls get a deeper pipeline.
static bool pf_fit(PfParams& p) {
    for (int st = 6; st >= 2; --st) {
        p.stages = st;
        p.raw_slots = 0;
        const size_t used = 1024 + (size_t)st * p.stage_bytes + pf_ctrl_bytes(p) + 64;
        if (used >= 232448) continue;
        const int r = (int)((232448 - used) / p.raw_slot_bytes);
        if (r >= 3 || st == 2) {
            p.raw_slots = r > 4 ? 4 : r;
            return p.raw_slots >= 1;
        }
    }
    return false;
}

// B rows a stage holds: a unit has at most min(T, kPfMaxN) columns (a token
// selects an expert at most once), rounded to the MMA's 16.
static uint32_t pf_stage_cols(int T) {
    const int n = (T + 15) & ~15;
    return (uint32_t)(n < kPfMaxN ? n : kPfMaxN);
}

template <int MODE>
static cudaError_t pf_launch_gemm(PfParams& p, int grid, cudaStream_t s) {
    const size_t bars = pf_ctrl_bytes(p);
    const size_t smem = 1024 + (size_t)p.stages * p.stage_bytes +
                        (size_t)p.raw_slots * p.raw_slot_bytes + bars;
    if (smem > 232448) return cudaErrorInvalidConfiguration;
    const cudaError_t attr = cudaFuncSetAttribute(
        k_pf_gemm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (attr != cudaSuccess) return attr;
    return pf_launch(p.T, k_pf_gemm<MODE>, dim3(grid), dim3(kPfThreads), smem, s, p);
}

// The warp-level MMA path for few tokens (k_bd_gemm): every side's gate and
// up share one block format (a lane decodes one format for its whole row
// tile).
static bool bd_supported(const moe_b200_layer* L, int T, bool routed, bool shared) {
    if (T > kBdMaxT) return false;
    if (routed && L->gate_type != L->up_type) return false;
    if (shared && L->shared_gate_type != L->shared_up_type) return false;
    if (routed && (L->intermediate % 128 || L->hidden % 256)) return false;
    if (shared && L->shared_intermediate % 128) return false;
    return true;
}

// Buffer bytes of k_bd_gemm: raw rows of the side with the widest boxes,
// rounded to 1 KB, plus the B tile (4 stages x kBdMaxN rows x 128 B).
static uint32_t bd_buf_bytes(const PfParams& g, int mode) {
    uint32_t best = 0;
    for (int sd = 0; sd < 2; ++sd) {
        const int w0 = pf_w(g.side[sd].type), w1 = pf_w(g.side[sd].type2);
        const uint32_t raw = mode == PF_GATEUP ? (uint32_t)(kBdRows / 2 * (w0 + w1)) : (uint32_t)(kBdRows * w0);
        const uint32_t b = ((raw + 1023u) & ~1023u) + 4u * kBdMaxN * 128u;
        best = b > best ? b : best;
    }
    return best;
}

template <int MODE>
static cudaError_t bd_launch(PfParams& p, int grid, cudaStream_t s) {
    p.stage_bytes = bd_buf_bytes(p, MODE);
    const size_t smem = 1024 + 2 * (size_t)p.stage_bytes + 8 * kBdWarpRows * 128 + 24 +
                        (size_t)2 * (p.n_routed + 1) * 4 + 16;
    if (smem > 232448) return cudaErrorInvalidConfiguration;
    const cudaError_t attr = cudaFuncSetAttribute(
        k_bd_gemm<MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (attr != cudaSuccess) return attr;
    return pf_launch(p.T, k_bd_gemm<MODE>, dim3(grid), dim3(kBdThreads), smem, s, p);
}

static int pf_fail(cudaError_t* ce, cudaError_t e) {
    if (ce) *ce = e;
    return ST_CUDA;
}

int prefill_run(const moe_b200_layer* L, const void* x, int x_bf16, int T, float* y,
                int32_t* ids_out, float* w_out, void* ws, size_t ws_bytes, cudaStream_t s,
                cudaError_t* ce) {
    const int flags = L->flags;
    if (!prefill_supported(L, flags)) return ST_TYPE;
    const PfWs W = pf_ws(L, T);
    if (ws_bytes < W.total) return ST_WORKSPACE;
    char* base = static_cast<char*>(ws);
    const bool routed = !(flags & MOE_B200_SHARED_ONLY);
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    const int H = L->hidden, E = L->n_experts, K = L->top_k;
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate
                                                              : L->intermediate;
    const int n_routed = routed ? L->expert_count : 0;
    const int sms = sm_count();
    uint32_t* err = reinterpret_cast<uint32_t*>(base + 32);

    PfPrep pp{};
    pp.T = T;
    pp.H = H;
    pp.E = E;
    pp.n_routed = n_routed;
    pp.x_bf16 = x_bf16;
    pp.x = x;
    pp.gate_inp = shared ? L->shared_gate_inp : nullptr;
    pp.router = L->router;
    pp.xh = reinterpret_cast<__half*>(base + W.xh);
    pp.xl = reinterpret_cast<__half*>(base + W.xl);
    pp.rh = reinterpret_cast<__half*>(base + W.rh);
    pp.rl = reinterpret_cast<__half*>(base + W.rl);
    pp.xs_inv = reinterpret_cast<float*>(base + W.xs_inv);
    pp.rs_inv = reinterpret_cast<float*>(base + W.rs_inv);
    pp.sg = reinterpret_cast<float*>(base + W.sg);
    pp.y = y;
    pp.counts = reinterpret_cast<int32_t*>(base + W.counts);
    pp.cursor = reinterpret_cast<int32_t*>(base + W.cursor);
    const bool small_router = routed && pf_small_router(L, T) && ((uintptr_t)x & 15u) == 0;
    pp.want_lo = routed && !small_router;
    cudaError_t e = pf_launch(T, k_pf_prep_x, dim3(T), dim3(256), 0, s, pp);
    if (e != cudaSuccess) return pf_fail(ce, e);

    PfParams gp{};
    gp.T = T;
    gp.H = H;
    gp.E = E;
    gp.Imax = Imax;
    gp.err = err;
    gp.xs_inv = pp.xs_inv;
    gp.rs_inv = pp.rs_inv;
    gp.sg = pp.sg;
    gp.y = y;
    gp.counts = pp.counts;
    gp.pair_tok = reinterpret_cast<int32_t*>(base + W.ptok);
    gp.pair_w = reinterpret_cast<float*>(base + W.pw);
    gp.act = reinterpret_cast<__half*>(base + W.act);
    gp.logits = reinterpret_cast<float*>(base + W.logits);
    gp.bias = L->router_bias;
    {
        int cap = 0;
        uint64_t* tb = trace_buffer(&cap);
        gp.trace = (tb && cap >= sms) ? tb : nullptr;
    }

    PfRoute rp{};
    rp.T = T;
    rp.E = E;
    rp.K = K;
    rp.expert_begin = L->expert_begin;
    rp.n_routed = n_routed;
    rp.logits = gp.logits;
    rp.ids = reinterpret_cast<int32_t*>(base + W.ids);
    rp.w = reinterpret_cast<float*>(base + W.w);
    rp.ids_out = ids_out;
    rp.w_out = w_out;
    rp.counts = pp.counts;
    rp.cursor = pp.cursor;
    rp.pair_tok = const_cast<int32_t*>(gp.pair_tok);
    rp.pair_w = const_cast<float*>(gp.pair_w);

    // the small router routes its tokens itself (up to 256 experts; arrival
    // counters in workspace bytes 128..255, control words that stay zero
    // between calls)
    const bool fused_topk = routed && small_router && E <= 256;
    if (routed && small_router) {
        uint32_t* tcnt = fused_topk ? reinterpret_cast<uint32_t*>(base + kRsCntOffset) : nullptr;
        e = pf_launch(T, k_pf_router_small, dim3((E + kRsE - 1) / kRsE, (T + kRsTok - 1) / kRsTok),
                      dim3(256), 0, s, pp, L->router_bias, gp.logits, rp, tcnt);
        if (e != cudaSuccess) return pf_fail(ce, e);
    } else if (routed) {
        if ((e = pf_launch(T, k_pf_prep_router, dim3(E), dim3(256), 0, s, pp)) != cudaSuccess)
            return pf_fail(ce, e);
        // router logits
        PfParams rp2 = gp;
        bool ok = make_map(&rp2.rmap[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.rh, H, E, (uint64_t)H * 2, 64, 128, true) &&
                  make_map(&rp2.rmap[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.rl, H, E, (uint64_t)H * 2, 64, 128, true) &&
                  make_map(&rp2.rbmap[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.xh, H, T, (uint64_t)H * 2, 64, 16, true) &&
                  make_map(&rp2.rbmap[1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.xl, H, T, (uint64_t)H * 2, 64, 16, true);
        if (!ok) return ST_INTERNAL;
        rp2.segs = 3;
        rp2.rchunks = kPfRouterChunks;
        rp2.rpart = reinterpret_cast<float*>(base + W.rpart);
        rp2.stages = 4;
        rp2.raw_slots = 0;
        rp2.a_bytes = 16384;
        rp2.stage_bytes = 16384 + kPfRouterN * 128;
        rp2.raw_slot_bytes = 0;
        rp2.n_routed = 0;
        rp.part = rp2.rpart;
        rp.nparts = rp2.rchunks;
        rp.bias = L->router_bias;
        const int units = ((E + 127) / 128) * ((T + kPfRouterN - 1) / kPfRouterN) * rp2.rchunks;
        if ((e = pf_launch_gemm<PF_ROUTER>(rp2, units < sms ? units : sms, s)) != cudaSuccess)
            return pf_fail(ce, e);
    }
    if (routed) {
        // more than 256 experts: each warp stages its scores in shared memory
        // (E floats + E flags), within the default 48 KB per block
        const size_t wsm = E > 256 ? ((size_t)E * 5 + 15) / 16 * 16 : 0;
        int wpb = kPfTopkWarps;
        while (wpb > 1 && (size_t)wpb * wsm > 48 * 1024) --wpb;
        if (!fused_topk &&
            (e = pf_launch(T, k_pf_topk, dim3((T + wpb - 1) / wpb), dim3(32 * wpb), (size_t)wpb * wsm,
                           s, rp)) != cudaSuccess)
            return pf_fail(ce, e);
        const __half* xh = pp.xh;
        __half* xperm = reinterpret_cast<__half*>(base + W.xperm);
        if ((e = pf_launch(T, k_pf_pairs, dim3((T * K + 7) / 8), dim3(256), 0, s, rp, xh, xperm, H)) !=
            cudaSuccess)
            return pf_fail(ce, e);
    }

    // expert GEMMs: warp-level MMA for few tokens, the tcgen05 pipeline otherwise
    const bool use_bd = bd_supported(L, T, routed, shared) && !(flags & MOE_B200_TCGEN05);
    gp.n_routed = n_routed;
    gp.has_shared = shared ? 1 : 0;
    const int act_rows = T * K + T;
    int wmax_gu = 0, wmax_dn = 0;
    // gate/up
    {
        PfParams g = gp;
        __half* xperm = reinterpret_cast<__half*>(base + W.xperm);
        const uint64_t prows = (uint64_t)T * K;
        bool ok = make_map(&g.bmap[0][0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xperm, H, prows, (uint64_t)H * 2, 64, 128, true) &&
                  make_map(&g.bmap[0][1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xperm, H, prows, (uint64_t)H * 2, 64, 16, true) &&
                  make_map(&g.bmap[1][0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.xh, H, T, (uint64_t)H * 2, 64, 128, true) &&
                  make_map(&g.bmap[1][1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, pp.xh, H, T, (uint64_t)H * 2, 64, 16, true);
        if (routed) {
            const int t0 = L->gate_type, t1 = L->up_type;
            const uint64_t rb0 = row_bytes(t0, H), rb1 = row_bytes(t1, H);
            const uint64_t rows = (uint64_t)n_routed * L->intermediate;
            ok = ok && make_map(&g.wmap[0][0], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->gate, rb0, rows, rb0, pf_w(t0), 64, false) &&
                 make_map(&g.wmap[0][1], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->up, rb1, rows, rb1, pf_w(t1), 64, false);
            g.side[0] = PfSide{t0, t1, L->intermediate, H};
            wmax_gu = pf_w(t0) + pf_w(t1);
        } else {
            g.side[0] = PfSide{Q8_0, Q8_0, 128, 256};
        }
        if (shared) {
            const int t0 = L->shared_gate_type, t1 = L->shared_up_type;
            const uint64_t rb0 = row_bytes(t0, H), rb1 = row_bytes(t1, H);
            ok = ok && make_map(&g.wmap[1][0], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->shared_gate, rb0, L->shared_intermediate, rb0, pf_w(t0), 64, false) &&
                 make_map(&g.wmap[1][1], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->shared_up, rb1, L->shared_intermediate, rb1, pf_w(t1), 64, false);
            g.side[1] = PfSide{t0, t1, L->shared_intermediate, H};
            const int tw = pf_w(t0) + pf_w(t1);
            wmax_gu = tw > wmax_gu ? tw : wmax_gu;
        } else {
            g.side[1] = PfSide{Q8_0, Q8_0, 128, 256};
        }
        if (!ok) return ST_INTERNAL;
        if (use_bd) {
            if ((e = bd_launch<PF_GATEUP>(g, kBdCtasPerSm * sms, s)) != cudaSuccess) return pf_fail(ce, e);
        } else {
            g.a_bytes = 16384;
            g.stage_bytes = g.a_bytes + pf_stage_cols(T) * 128;
            g.raw_slot_bytes = 64 * wmax_gu;
            if (!pf_fit(g)) return ST_INTERNAL;
            if ((e = pf_launch_gemm<PF_GATEUP>(g, sms, s)) != cudaSuccess) return pf_fail(ce, e);
        }
    }
    // down
    {
        PfParams g = gp;
        bool ok = make_map(&g.bmap[0][0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, gp.act, Imax, act_rows, (uint64_t)Imax * 2, 64, 128, true) &&
                  make_map(&g.bmap[0][1], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, gp.act, Imax, act_rows, (uint64_t)Imax * 2, 64, 16, true);
        g.bmap[1][0] = g.bmap[0][0];
        g.bmap[1][1] = g.bmap[0][1];
        if (routed) {
            const int tw = pf_w(L->down_type);
            const uint64_t rb = row_bytes(L->down_type, L->intermediate);
            ok = ok && make_map(&g.wmap[0][0], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->down, rb, (uint64_t)n_routed * H, rb, tw, 128, false);
            g.side[0] = PfSide{L->down_type, L->down_type, H, L->intermediate};
            wmax_dn = tw;
        } else {
            g.side[0] = PfSide{Q8_0, Q8_0, 128, 256};
        }
        if (shared) {
            const int tw = pf_w(L->shared_down_type);
            const uint64_t rb = row_bytes(L->shared_down_type, L->shared_intermediate);
            ok = ok && make_map(&g.wmap[1][0], CU_TENSOR_MAP_DATA_TYPE_UINT8, L->shared_down, rb, H, rb, tw, 128, false);
            g.side[1] = PfSide{L->shared_down_type, L->shared_down_type, H, L->shared_intermediate};
            wmax_dn = tw > wmax_dn ? tw : wmax_dn;
        } else {
            g.side[1] = PfSide{Q8_0, Q8_0, 128, 256};
        }
        if (!ok) return ST_INTERNAL;
        if (use_bd) {
            if ((e = bd_launch<PF_DOWN>(g, kBdCtasPerSm * sms, s)) != cudaSuccess) return pf_fail(ce, e);
        } else {
            g.a_bytes = 16384;
            g.stage_bytes = g.a_bytes + pf_stage_cols(T) * 128;
            g.raw_slot_bytes = 128 * wmax_dn;
            if (!pf_fit(g)) return ST_INTERNAL;
            if ((e = pf_launch_gemm<PF_DOWN>(g, sms, s)) != cudaSuccess) return pf_fail(ce, e);
        }
    }
    return ST_OK;
}

int prefill_kernels(const moe_b200_layer* L, int T) {
    const bool routed = !(L->flags & MOE_B200_SHARED_ONLY);
    if (!routed) return 3;
    // prep, router (small: with the top-k when E <= 256; else prep_router,
    // router GEMM, top-k), pairs, gate/up, down
    if (pf_small_router(L, T)) return L->n_experts <= 256 ? 5 : 6;
    return 7;
}

}  // namespace moeb200
