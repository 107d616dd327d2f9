// topk.cuh -- top-k selection and routing weights of one token, one warp.
//
// Same selection and arithmetic as ExpertRouter.route (reference
// src/flash_moe/router.py:151-170): the k highest scores in descending order
// (ties to the lower expert id), a float64 softmax over those k only with
// numpy's summation order for the denominator (np.add.reduce pairwise sum),
// uniform weights if the sum is not finite or not positive, and the weights
// rounded to fp32 as numpy rounds a Python float multiplying an fp32 array.
#pragma once

#include <math.h>

#include "common.cuh"
#include "sm100.cuh"

namespace moeb200 {

constexpr int kMaxTopK = 16;

// numpy's pairwise summation of n <= 128 float64 values: sequential from 0
// below 8, eight interleaved partial sums combined as
// ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) from 8 on.
__device__ __forceinline__ double np_sum(const double* v, int n) {
    if (n < 8) {
        double r = 0.0;
        for (int i = 0; i < n; ++i) r += v[i];
        return r;
    }
    double r[8];
    for (int j = 0; j < 8; ++j) r[j] = v[j];
    int i = 8;
    for (; i < n - (n % 8); i += 8)
        for (int j = 0; j < 8; ++j) r[j] += v[i + j];
    double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; ++i) res += v[i];
    return res;
}

// scores: E floats in shared memory; taken: E bytes of shared scratch.
// Writes ids[K] / w[K] (lane 0).  All 32 lanes must call.
static __device__ __noinline__ void topk_softmax_warp(const float* scores, unsigned char* taken, int E,
                                                  int K, int* ids, float* w) {
    const int lane = threadIdx.x & 31;
    for (int e = lane; e < E; e += 32) taken[e] = 0;
    __syncwarp();
    float sel_v[kMaxTopK];
    int sel_i[kMaxTopK];
    for (int k = 0; k < K; ++k) {
        float best = -INFINITY;
        int bi = 0x7fffffff;
        for (int e = lane; e < E; e += 32) {
            const float v = scores[e];
            if (!taken[e] && (bi == 0x7fffffff || v > best || (v == best && e < bi))) {
                best = v;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > best || (ov == best && oi < bi))) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) taken[bi] = 1;
        __syncwarp();
        sel_v[k] = best;
        sel_i[k] = bi;
    }
    if (lane == 0 && K > 0) {
        double m = (double)sel_v[0];
        for (int k = 1; k < K; ++k) m = fmax(m, (double)sel_v[k]);
        double ex[kMaxTopK];
        for (int k = 0; k < K; ++k) ex[k] = exp((double)sel_v[k] - m);
        const double tot = np_sum(ex, K);
        const bool uniform = !isfinite(tot) || tot <= 0.0;
        for (int k = 0; k < K; ++k) {
            ids[k] = sel_i[k];
            w[k] = uniform ? (float)(1.0 / K) : (float)(ex[k] / tot);
        }
    }
    __syncwarp();
}

// Order-preserving map of an fp32 value to a uint32 key (larger value ->
// larger key); NaN maps above +inf, as numpy's argsort places it last.
__device__ __forceinline__ uint32_t fkey(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float fkey_inv(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// (key, id) a sorts before b: larger key, then lower id.
__device__ __forceinline__ bool kbefore(uint32_t ka, int ia, uint32_t kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

#define MOE_CSWAP(a, b)                                                  \
    do {                                                                 \
        if (kbefore(k[b], id[b], k[a], id[a])) {                         \
            const uint32_t tk = k[a]; k[a] = k[b]; k[b] = tk;            \
            const int ti = id[a]; id[a] = id[b]; id[b] = ti;             \
        }                                                                \
    } while (0)

// Top-k of E <= 256 keys held 8 per lane (lane l: experts 8l..8l+7, absent
// ones key 0 / id 0x7fffffff).  Each lane sorts its keys in registers; each
// of the K rounds takes the warp maximum of the lane heads with one
// redux.sync, and the winning lane pops its head.  Lane r (r < K) ends with
// selection r: its key in my_k, its expert in my_id.
__device__ __forceinline__ void topk_select_warp(uint32_t (&k)[8], int (&id)[8], int K,
                                                 uint32_t& my_k, int& my_id,
                                                 uint64_t* trace = nullptr) {
    const int lane = threadIdx.x & 31;
    // Batcher odd-even merge sort of 8, descending (19 compare-exchanges)
    MOE_CSWAP(0, 1); MOE_CSWAP(2, 3); MOE_CSWAP(4, 5); MOE_CSWAP(6, 7);
    MOE_CSWAP(0, 2); MOE_CSWAP(1, 3); MOE_CSWAP(4, 6); MOE_CSWAP(5, 7);
    MOE_CSWAP(1, 2); MOE_CSWAP(5, 6);
    MOE_CSWAP(0, 4); MOE_CSWAP(1, 5); MOE_CSWAP(2, 6); MOE_CSWAP(3, 7);
    MOE_CSWAP(2, 4); MOE_CSWAP(3, 5);
    MOE_CSWAP(1, 2); MOE_CSWAP(3, 4); MOE_CSWAP(5, 6);
    if (trace && lane == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        trace[13] = t;
    }
    my_k = 0;
    my_id = 0;
    for (int r = 0; r < K; ++r) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, k[0]);
        // equal keys: lower lane holds lower ids; within a lane the sort
        // already put the lower id first
        const uint32_t ball = __ballot_sync(0xffffffffu, k[0] == m);
        const int win = __ffs(ball) - 1;
        const int wid = __shfl_sync(0xffffffffu, id[0], win);
        if (lane == r) {
            my_k = m;
            my_id = wid;
        }
        if (lane == win) {
#pragma unroll
            for (int i = 0; i < 7; ++i) {
                k[i] = k[i + 1];
                id[i] = id[i + 1];
            }
            k[7] = 0u;
            id[7] = 0x7fffffff;
        }
    }
    if (trace && lane == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        trace[14] = t;
    }
}

// Routing weights of the K selections lanes 0..K-1 hold (topk_select_warp):
// the float64 softmax over those k only (router.py:158-168), written to
// ids[lane] / w[lane].  All 32 lanes must call.
__device__ __forceinline__ void topk_weights_warp(uint32_t my_k, int my_id, int K, int* ids,
                                                  float* w) {
    const int lane = threadIdx.x & 31;
    const double v = (lane < K) ? (double)fkey_inv(my_k) : 0.0;
    const double mx = __shfl_sync(0xffffffffu, v, 0);  // selection 0 is the maximum
    const double ex = (lane < K) ? exp(v - mx) : 0.0;
    double tot;
    if (K == 8) {
        // numpy's 8-wide pairwise sum ((e0+e1)+(e2+e3))+((e4+e5)+(e6+e7))
        double t = ex + __shfl_xor_sync(0xffffffffu, ex, 1);
        t = t + __shfl_xor_sync(0xffffffffu, t, 2);
        t = t + __shfl_xor_sync(0xffffffffu, t, 4);
        tot = __shfl_sync(0xffffffffu, t, 0);
    } else {
        double all[kMaxTopK];
        for (int i = 0; i < K; ++i) all[i] = __shfl_sync(0xffffffffu, ex, i);
        tot = np_sum(all, K);
    }
    if (lane < K) {
        const bool uniform = !isfinite(tot) || tot <= 0.0;
        ids[lane] = my_id;
        w[lane] = uniform ? (float)(1.0 / K) : (float)(ex / tot);
    }
    __syncwarp();
}

// Compact top-k of E <= 256 keys held 8 per lane (lane l: experts
// 8l..8l+7, absent ones key 0 / id 0x7fffffff), for kernels whose whole
// step must stay small in the instruction cache: K rounds of a warp
// arg-max over (key, lower id first) composites, the winner cleared where
// it sits.  Same selection, in the same order, as topk_select_warp.  Lane r
// (r < K) ends with selection r: its key in my_k, its expert in my_id.
__device__ __forceinline__ void topk_select_compact(const uint32_t (&k)[8], const int (&id)[8],
                                                    int K, uint32_t& my_k, int& my_id) {
    const int lane = threadIdx.x & 31;
    uint64_t cmp[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) cmp[i] = ((uint64_t)k[i] << 32) | (uint32_t)~(uint32_t)id[i];
    my_k = 0;
    my_id = 0;
#pragma unroll 1
    for (int r = 0; r < K; ++r) {
        uint64_t b = cmp[0];
#pragma unroll
        for (int i = 1; i < 8; ++i) b = cmp[i] > b ? cmp[i] : b;
        const uint32_t bh = (uint32_t)(b >> 32);
        const uint32_t m = __reduce_max_sync(0xffffffffu, bh);
        const uint32_t ml = __reduce_max_sync(0xffffffffu, bh == m ? (uint32_t)b : 0u);
        const uint64_t win = ((uint64_t)m << 32) | ml;
        if (lane == r) {
            my_k = m;
            my_id = (int)~ml;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) cmp[i] = cmp[i] == win ? 0ull : cmp[i];
    }
}

// Routing weights of the K selections lanes 0..K-1 hold, in fp32: the
// softmax over those k only (router.py:158-168; the reference's float64
// weights differ from these by about one fp32 ulp), uniform weights when
// the sum is not finite or not positive.  Written to ids[lane] / w[lane].
// All 32 lanes must call.
__device__ __forceinline__ void topk_weights_f32(uint32_t my_k, int my_id, int K, int* ids, float* w) {
    const int lane = threadIdx.x & 31;
    const float v = lane < K ? fkey_inv(my_k) : 0.f;
    const float mx = __shfl_sync(0xffffffffu, v, 0);  // selection 0 is the maximum
    const float ex = lane < K ? expf(v - mx) : 0.f;
    float tot = ex;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
    if (lane < K) {
        const bool uniform = !isfinite(tot) || tot <= 0.f;
        ids[lane] = my_id;
        w[lane] = uniform ? 1.0f / (float)K : ex / tot;
    }
    __syncwarp();
}

// Fast form of topk_softmax_warp for E <= 256 with the scores in global
// memory written by other CTAs (read through L2).  Identical results to
// topk_softmax_warp.
__device__ __forceinline__ void topk_softmax_warp_fast(const float* gscores, int E, int K,
                                                       int* ids, float* w,
                                                       uint64_t* trace = nullptr) {
    const int lane = threadIdx.x & 31;
    uint32_t k[8];
    int id[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = 8 * lane + i;
        k[i] = e < E ? fkey(__ldcg(gscores + e)) : 0u;
        id[i] = e < E ? e : 0x7fffffff;
    }
    uint32_t my_k;
    int my_id;
    topk_select_warp(k, id, K, my_k, my_id, trace);
    topk_weights_warp(my_k, my_id, K, ids, w);
    if (trace && lane == 0) {
        uint64_t t;
        asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
        trace[15] = t;
    }
}

// Lane l's keys for topk_select_warp (experts 8l..8l+7 of E <= 256) from
// exchange words (st_word_gpu: the fp32 score and the step tag in one 64-bit
// word), polled until every one of the first S >= E words carries `tag`
// (words E..S-1 carry no score: they only show that their writer has reached
// this step).  The polling loads are coalesced: lane l reads words l + 32 i,
// so a warp's load is 256 contiguous bytes -- every CTA of the grid polls
// the same words, and the sectors per round are what the L2 slices serve.
// Only the words still missing are read again.  The keys are staged in
// shared memory (`stage`, S uint32) and each lane then takes its own
// experts from there.  At most `limit` rounds; false (the same in every
// lane) when it gave up.  S <= 256.
__device__ __forceinline__ bool load_score_words(const uint64_t* words, int E, int S, uint32_t tag,
                                                 uint32_t limit, uint32_t* stage,
                                                 uint32_t (&k)[8], int (&id)[8]) {
    const int lane = threadIdx.x & 31;
    uint32_t pend = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i)
        if (lane + 32 * i < S) pend |= 1u << i;
    bool ok = true;
    for (uint32_t round = 0; __any_sync(0xffffffffu, pend != 0u); ++round) {
        if (round == limit) {
            ok = false;
            break;
        }
        uint64_t wv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) wv[i] = (pend >> i) & 1u ? ld_word_gpu(words + lane + 32 * i) : 0ull;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            if (((pend >> i) & 1u) && (uint32_t)(wv[i] >> 32) == tag) {
                stage[lane + 32 * i] = fkey(__uint_as_float((uint32_t)wv[i]));
                pend &= ~(1u << i);
            }
        }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = 8 * lane + i;
        id[i] = e < E ? e : 0x7fffffff;
        k[i] = e < E ? stage[e] : 0u;
    }
    __syncwarp();
    return ok;
}

#undef MOE_CSWAP

// sigmoid of the reference shared-expert gate (shared_expert.py:55-62).
__device__ __forceinline__ float shared_sigmoid(float v) {
    if (v >= 0.f) return 1.0f / (1.0f + expf(-v));
    const float e = expf(v);
    return e / (1.0f + e);
}

}  // namespace moeb200
