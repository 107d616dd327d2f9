// decode.cu -- fused single-token MoE layer decode (the fast engine).
//
// One cooperative launch, one CTA per SM, computes the whole layer for one
// token: router scores -> top-k + softmax -> routed SwiGLU gate/up -> down ->
// weighted sum + sigmoid-gated shared expert (reference run_moe_layer,
// src/flash_moe/moe_layer.py:39-107, with moe_quant_expert,
// cpp/moe_quant_dot.cpp:171-214, for each selected expert).
//
// Work split over G CTAs (c = blockIdx.x), all static except the routed part:
//   router rows       [E*c/G, E*(c+1)/G)
//   shared gate/up    rows [Is*c/G, Is*(c+1)/G)
//   output rows       [H*c/G, H*(c+1)/G) of the shared and every routed down
//   routed gate/up    flattened (slot, row) range [A*I*c/G, A*I*(c+1)/G),
//                     A = number of selected experts this GPU holds
// so every CTA moves ~1/G of the layer's bytes.  Its packed rows are copied
// HBM -> shared memory with one-dimensional TMA bulk copies (cp.async.bulk,
// no multicast): the router and shared-expert rows at kernel entry, the
// routed rows as soon as the CTA knows the routing.  Phases synchronise
// through release/acquire counters in the workspace (bounded waits; a wait
// that gives up records -9 in the workspace error word and the kernel runs
// on to its end).  The last CTA to finish resets the counters, so the
// workspace is ready for the next launch on the same stream.
//
// The routing is recomputed identically by every CTA from the E scores, so
// no CTA waits for another to publish it.  Exchanges through global memory:
// E scores, the A*I + Is fp32 activations, the shared gate value.
#include <math.h>
#include <stdlib.h>

#include "launch.h"
#include "qdot.cuh"
#include "sm100.cuh"
#include "topk.cuh"

namespace moeb200 {

constexpr int kFusedThreads = 512;
constexpr uint32_t kWaitPolls = 1u << 21;
constexpr int kTraceSlots = 32;
constexpr int kMaxChunks = 8;  // routed gate/up copy chunks (mbarriers 3..10)

enum { C_ROUTER = 0, C_SHARED = 1, C_GATEUP = 2, C_EXIT = 3, C_ERROR = 8 };

struct FusedParams {
    moe_b200_layer L;
    const float* x;
    float* y;
    int32_t* ids_out;
    float* w_out;
    uint32_t* ctr;   // counters, error word at ctr[C_ERROR]
    float* scores;   // [E]
    float* act_r;    // [K x I]
    float* act_s;    // [Is]
    float* sg;       // [1]
    uint64_t* trace; // [G x 16] phase timestamps (ns), or null
    int G;
    int with_shared;
    int max_router_rows, max_sgu_rows, max_out_rows, max_rgu_rows;
    int lpr_h, lpr_i, lpr_is;
    int chunk_rows;
    int warm;
    uint32_t o_x32, o_xq, o_router, o_sgate, o_sup, o_sdown, o_rgate, o_rup, o_rdown;
    uint32_t o_act, o_aq, o_misc, total;
};

__device__ __forceinline__ int part(int n, int c, int G) { return (int)(((int64_t)n * c) / G); }

__device__ __forceinline__ void set_error(uint32_t* ctr, int code) {
    atomicExch(reinterpret_cast<int*>(ctr + C_ERROR), code);
}

// fp32 row dot with x in shared memory, one warp.
__device__ __forceinline__ float dot_f32_warp(const float* row, const float* x, int n, int lane) {
    float acc = 0.f;
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const float4* x4 = reinterpret_cast<const float4*>(x);
    for (int i = lane; i < (n >> 2); i += 32) {
        const float4 a = r4[i], b = x4[i];
        acc = fmaf(a.x, b.x, acc);
        acc = fmaf(a.y, b.y, acc);
        acc = fmaf(a.z, b.z, acc);
        acc = fmaf(a.w, b.w, acc);
    }
    return warp_sum(acc);
}

// GU: gate and up type, DN: routed down type, SGU: shared gate and up type,
// SDN: shared down type -- each a ggml type id fixed at compile time, or -1
// to dispatch on the layer's runtime types (the generic instance).
template <int GU, int DN, int SGU, int SDN>
__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_fused(const __grid_constant__ FusedParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const moe_b200_layer& L = p.L;
    const int c = blockIdx.x, G = p.G, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = kFusedThreads / 32;
    const int H = L.hidden, I = L.intermediate, E = L.n_experts, K = L.top_k;
    const int Is = p.with_shared ? L.shared_intermediate : 0;
    const int64_t rb_gate = row_bytes(L.gate_type, H), rb_up = row_bytes(L.up_type, H);
    const int64_t rb_down = row_bytes(L.down_type, I);
    const int64_t st_gate = rb_gate * I, st_up = rb_up * I, st_down = rb_down * H;
    const int64_t rb_sg = Is ? row_bytes(L.shared_gate_type, H) : 0;
    const int64_t rb_su = Is ? row_bytes(L.shared_up_type, H) : 0;
    const int64_t rb_sd = Is ? row_bytes(L.shared_down_type, Is) : 0;

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + p.o_misc);       // [3 + kMaxChunks]
    int* s_ids = reinterpret_cast<int*>(sm + p.o_misc + 128);          // [16]
    float* s_w = reinterpret_cast<float*>(sm + p.o_misc + 192);        // [16]
    int* s_act = reinterpret_cast<int*>(sm + p.o_misc + 256);          // [16] active slots
    int* s_nact = reinterpret_cast<int*>(sm + p.o_misc + 320);
    float* s_sg = reinterpret_cast<float*>(sm + p.o_misc + 324);
    float* s_part = reinterpret_cast<float*>(sm + p.o_misc + 384);     // [32] router partials
    float* s_scores = reinterpret_cast<float*>(sm + p.o_misc + 512);   // [E]
    unsigned char* s_taken = reinterpret_cast<unsigned char*>(s_scores + E);
    float* s_vout = reinterpret_cast<float*>(sm + p.o_misc + 512 + ((5 * E + 15) & ~15));

    const int r0 = part(E, c, G), r1 = part(E, c + 1, G);
    const int s0 = part(Is, c, G), s1 = part(Is, c + 1, G);
    const int h0 = part(H, c, G), h1 = part(H, c + 1, G);
    const int nh = h1 - h0;
    uint64_t* trace = p.trace ? p.trace + (size_t)c * kTraceSlots : nullptr;
#define TRACE(i) do { if (trace && tid == 0) trace[i] = global_ns(); } while (0)
    TRACE(0);

    if (tid == 0) {
        for (int i = 0; i < 3 + kMaxChunks; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    // ---- phase-0 copies: router rows, shared gate/up rows, shared down rows
    if (tid == 0) {
        uint32_t bytes = (uint32_t)((r1 - r0) * H * 4);
        if (Is) bytes += (uint32_t)((s1 - s0) * (rb_sg + rb_su) + nh * rb_sd);
        mbar_arrive_expect_tx(&bars[0], bytes);
        if (r1 > r0)
            bulk_g2s(sm + p.o_router, L.router + (size_t)r0 * H, (uint32_t)((r1 - r0) * H * 4), &bars[0]);
        if (Is && s1 > s0) {
            bulk_g2s(sm + p.o_sgate, L.shared_gate + s0 * rb_sg, (uint32_t)((s1 - s0) * rb_sg), &bars[0]);
            bulk_g2s(sm + p.o_sup, L.shared_up + s0 * rb_su, (uint32_t)((s1 - s0) * rb_su), &bars[0]);
        }
        if (Is && nh > 0)
            bulk_g2s(sm + p.o_sdown, L.shared_down + h0 * rb_sd, (uint32_t)(nh * rb_sd), &bars[0]);
    }
    // ---- the token, fp32 and quantised
    float* x32 = reinterpret_cast<float*>(sm + p.o_x32);
    for (int i = tid; i < H; i += kFusedThreads) x32[i] = p.x[i];
    __syncthreads();
    const QVec xq = qvec_at(sm + p.o_xq, H);
    for (int b = warp; b < H / 256; b += nw) quantize_block_warp(x32, xq, b);
    __syncthreads();
    TRACE(1);
    if (Is && c == 0 && warp == 0) {
        float acc = 0.f;
        for (int i = lane; i < H; i += 32) acc = fmaf(x32[i], L.shared_gate_inp[i], acc);
        acc = warp_sum(acc);
        if (lane == 0) p.sg[0] = shared_sigmoid(acc);
    }
    // lane -> (row-in-warp, pair) for H-long rows
    const int lpr_h = p.lpr_h, sub_h = lane / lpr_h, pr_h = lane % lpr_h;
    XLane xl;
    load_xlane(xl, xq, pr_h >> 2, pr_h & 3);

    // ---- instruction-cache warm-up while the first copies are in flight.
    // Each kernel launch runs its critical-path code once per CTA, so every
    // phase would otherwise start on cold instruction caches.  Here the
    // decoders and the top-k run once on dummy data (4 warps per region, one
    // per SM sub-partition); their results feed a store guarded by a
    // condition that never holds (G > 0), so nothing is written.
    if (p.warm) {
        float dummy = 0.f;
        const uint8_t* junk = sm + p.o_x32;
        const int region = warp >> 2;
        if (region == 0) {
            dummy = qdot_t<GU>(L.gate_type, junk, 0, lane & 3, xl);
        } else if (region == 1) {
            dummy = qdot_t<DN>(L.down_type, junk, 0, lane & 3, xl);
        } else if (region == 2) {
            if (Is)
                dummy = qdot_t<SGU>(L.shared_gate_type, junk, 0, lane & 3, xl) +
                        qdot_t<SDN>(L.shared_down_type, junk, 0, lane & 3, xl);
        } else if (E <= 256) {
            int di[kMaxTopK];
            float dw[kMaxTopK];
            topk_softmax_warp_fast(p.scores, E, K, di, dw);
            dummy = dw[lane % K] + (float)di[lane % K];
        }
        dummy = group_sum(dummy, 32);
        if (G < 0 && dummy == 1.2345f) p.y[0] = dummy;
    }

    if (!mbar_wait(&bars[0], 0, kWaitPolls) && tid == 0) set_error(p.ctr, ST_TIMEOUT);
    __syncthreads();
    TRACE(2);

    // ---- router scores: each of the CTA's R rows is split over nw/R warps,
    // partial sums combined in a fixed order (deterministic)
    {
        const float* router_s = reinterpret_cast<const float*>(sm + p.o_router);
        const int R = r1 - r0;
        if (R > 0 && R <= nw) {
            const int spr = nw / R;
            const int row = warp / spr, sl = warp % spr;
            if (row < R) {
                const int cw = (H / spr) & ~3;  // 16-byte aligned slices
                const int c0 = sl * cw, cn = (sl == spr - 1) ? H - c0 : cw;
                float acc = dot_f32_warp(router_s + (size_t)row * H + c0, x32 + c0, cn, lane);
                if (lane == 0) s_part[warp] = acc;
            }
            __syncthreads();
            if (tid < R) {
                float acc = 0.f;
                for (int q = 0; q < spr; ++q) acc += s_part[tid * spr + q];
                if (L.router_bias) acc = __fadd_rn(acc, L.router_bias[r0 + tid]);
                p.scores[r0 + tid] = acc;
            }
        } else {
            for (int rr = warp; rr < R; rr += nw) {
                float acc = dot_f32_warp(router_s + (size_t)rr * H, x32, H, lane);
                if (lane == 0) {
                    if (L.router_bias) acc = __fadd_rn(acc, L.router_bias[r0 + rr]);
                    p.scores[r0 + rr] = acc;
                }
            }
        }
    }
    __syncthreads();
    if (tid == 0) red_release_add(p.ctr + C_ROUTER, 1);
    TRACE(3);

    // ---- shared expert gate/up (x is the token)
    if (Is) {
        const int rpw = 32 / lpr_h;
        for (int rb = warp * rpw; rb < s1 - s0; rb += nw * rpw) {
            const int rr = rb + sub_h;
            const bool ok = rr < s1 - s0;
            const int rs = ok ? rr : 0;
            float g = qdot_t<SGU>(L.shared_gate_type, sm + p.o_sgate + rs * rb_sg, pr_h >> 2, pr_h & 3, xl);
            float u = qdot_t<SGU>(L.shared_up_type, sm + p.o_sup + rs * rb_su, pr_h >> 2, pr_h & 3, xl);
            g = group_sum(g, lpr_h);
            u = group_sum(u, lpr_h);
            if (ok && pr_h == 0) p.act_s[s0 + rr] = (g * shared_sigmoid(g)) * u;
        }
    }
    __syncthreads();
    if (tid == 0) red_release_add(p.ctr + C_SHARED, 1);
    TRACE(4);

    // ---- routing (every CTA, identically)
    if (tid == 0 && !wait_flag(p.ctr + C_ROUTER, (uint32_t)G, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
    __syncthreads();
    TRACE(5);
    if (E > 256) {
        for (int e = tid; e < E; e += kFusedThreads) s_scores[e] = __ldcg(p.scores + e);
        __syncthreads();
    }
    if (warp == 0) {
        if (E <= 256)
            topk_softmax_warp_fast(p.scores, E, K, s_ids, s_w, trace);
        else
            topk_softmax_warp(s_scores, s_taken, E, K, s_ids, s_w);
        if (lane == 0) {
            int na = 0;
            for (int k = 0; k < K; ++k) {
                const int e = s_ids[k];
                if (e >= L.expert_begin && e < L.expert_begin + L.expert_count) s_act[na++] = k;
            }
            *s_nact = na;
            if (c == 0) {
                for (int k = 0; k < K; ++k) {
                    if (p.ids_out) p.ids_out[k] = s_ids[k];
                    if (p.w_out) p.w_out[k] = s_w[k];
                }
            }
        }
    }
    __syncthreads();
    TRACE(6);
    const int A = *s_nact;
    const int f0 = part(A * I, c, G), f1 = part(A * I, c + 1, G);

    // ---- phase-1 copies: routed gate/up rows of [f0, f1) in chunks of CR
    // rows (one mbarrier each, issued in order so compute can start on the
    // first chunk), then the routed down rows
    const int nrows = f1 - f0;
    const int CR = p.chunk_rows;
    if (tid == 0) {
        for (int q = 0; q * CR < nrows; ++q) {
            const int q0 = q * CR, q1 = min(nrows, q0 + CR);
            mbar_arrive_expect_tx(&bars[3 + q], (uint32_t)((q1 - q0) * (rb_gate + rb_up)));
            for (int f = f0 + q0; f < f0 + q1;) {
                const int a = f / I, r = f % I;
                const int n = min(f0 + q1 - f, I - r);
                const int64_t e = s_ids[s_act[a]] - L.expert_begin;
                bulk_g2s(sm + p.o_rgate + (int64_t)(f - f0) * rb_gate, L.gate + e * st_gate + r * rb_gate,
                         (uint32_t)(n * rb_gate), &bars[3 + q]);
                bulk_g2s(sm + p.o_rup + (int64_t)(f - f0) * rb_up, L.up + e * st_up + r * rb_up,
                         (uint32_t)(n * rb_up), &bars[3 + q]);
                f += n;
            }
        }
        mbar_arrive_expect_tx(&bars[2], (uint32_t)(A * nh * rb_down));
        if (nh > 0) {
            for (int a = 0; a < A; ++a) {
                const int64_t e = s_ids[s_act[a]] - L.expert_begin;
                bulk_g2s(sm + p.o_rdown + (int64_t)a * p.max_out_rows * rb_down,
                         L.down + e * st_down + h0 * rb_down, (uint32_t)(nh * rb_down), &bars[2]);
            }
        }
    }

    // ---- routed gate/up, chunk by chunk
    {
        const int rpw = 32 / lpr_h;
        int waited = -1;
        for (int rb = warp * rpw; rb < nrows; rb += nw * rpw) {
            const int qlast = min(rb + rpw - 1, nrows - 1) / CR;
            while (waited < qlast) {
                ++waited;
                if (!mbar_wait(&bars[3 + waited], 0, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
                if (waited < 2) TRACE(16 + waited);
            }
            const int rr = rb + sub_h;
            const bool ok = rr < nrows;
            const int rs = ok ? rr : 0;
            float g = qdot_t<GU>(L.gate_type, sm + p.o_rgate + rs * rb_gate, pr_h >> 2, pr_h & 3, xl);
            float u = qdot_t<GU>(L.up_type, sm + p.o_rup + rs * rb_up, pr_h >> 2, pr_h & 3, xl);
            g = group_sum(g, lpr_h);
            u = group_sum(u, lpr_h);
            if (ok && pr_h == 0) {
                const float sgm = 1.0f / (1.0f + expf(-g));
                p.act_r[f0 + rr] = (g * sgm) * u;
            }
            if (rb == 0) TRACE(18);
        }
        // every chunk barrier must have completed before the CTA moves on
        // (its copies write shared memory)
        for (int q = waited + 1; q * CR < nrows; ++q)
            if (!mbar_wait(&bars[3 + q], 0, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
    }
    TRACE(7);
    __syncthreads();
    TRACE(8);
    if (tid == 0) {
        red_release_add(p.ctr + C_GATEUP, 1);
        if (Is && !wait_flag(p.ctr + C_SHARED, (uint32_t)G, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        if (!wait_flag(p.ctr + C_GATEUP, (uint32_t)G, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
    }
    __syncthreads();
    TRACE(9);

    // ---- activations of the A routed experts (+ shared), quantised
    const int nvec = A + (Is ? 1 : 0);
    const int Imax = max(I, Is);
    float* act32 = reinterpret_cast<float*>(sm + p.o_act);
    for (int i = tid; i < (A * I) / 4; i += kFusedThreads) {
        const int e = 4 * i;
        *reinterpret_cast<float4*>(act32 + (e / I) * Imax + (e % I)) =
            __ldcg(reinterpret_cast<const float4*>(p.act_r) + i);
    }
    if (Is) {
        for (int i = tid; i < Is / 4; i += kFusedThreads)
            *reinterpret_cast<float4*>(act32 + A * Imax + 4 * i) =
                __ldcg(reinterpret_cast<const float4*>(p.act_s) + i);
        if (tid == 0) *s_sg = __ldcg(p.sg);
    }
    __syncthreads();
    TRACE(19);
    const uint32_t qb = qvec_bytes(Imax);
    {
        const int bi = I / 256, bs = Is / 256;
        for (int it = warp; it < A * bi + bs; it += nw) {
            const int v = it < A * bi ? it / bi : A;
            const int b = it < A * bi ? it % bi : it - A * bi;
            const int n = v < A ? I : Is;
            quantize_block_warp(act32 + v * Imax, qvec_at(sm + p.o_aq + v * qb, n), b);
        }
    }
    __syncthreads();
    TRACE(20);
    if (!mbar_wait(&bars[2], 0, kWaitPolls) && tid == 0) set_error(p.ctr, ST_TIMEOUT);
    __syncthreads();
    TRACE(10);

    // ---- down rows [h0, h1) of every vector: item = (vector, pair of row
    // groups); the activation codes are loaded once per item
    {
        const int rpw_i = 32 / p.lpr_i, rpw_s = 32 / p.lpr_is;
        const int ng_i = (nh + rpw_i - 1) / rpw_i, ng_s = Is ? (nh + rpw_s - 1) / rpw_s : 0;
        const int np_i = (ng_i + 1) / 2, np_s = (ng_s + 1) / 2;
        for (int it = warp; it < A * np_i + np_s; it += nw) {
            const bool sh = it >= A * np_i;
            const int v = sh ? A : it / np_i;
            const int gp = sh ? it - A * np_i : it % np_i;
            const int lpr = sh ? p.lpr_is : p.lpr_i;
            const int ng = sh ? ng_s : ng_i;
            const int rpw = 32 / lpr, sub = lane / lpr, pr = lane % lpr;
            const int type = sh ? L.shared_down_type : L.down_type;
            const int64_t rb = sh ? rb_sd : rb_down;
            const uint8_t* rows = sh ? sm + p.o_sdown : sm + p.o_rdown + (int64_t)v * p.max_out_rows * rb_down;
            const int n = sh ? Is : I;
            XLane xa;
            load_xlane(xa, qvec_at(sm + p.o_aq + v * qb, n), pr >> 2, pr & 3);
#pragma unroll
            for (int gg = 0; gg < 2; ++gg) {
                const int gi = 2 * gp + gg;
                if (gi < ng) {
                    const int rr = gi * rpw + sub;
                    const bool ok = rr < nh;
                    const uint8_t* rowp = rows + (ok ? rr : 0) * rb;
                    float d = sh ? qdot_t<SDN>(type, rowp, pr >> 2, pr & 3, xa)
                                 : qdot_t<DN>(type, rowp, pr >> 2, pr & 3, xa);
                    d = group_sum(d, lpr);
                    if (ok && pr == 0) s_vout[v * p.max_out_rows + rr] = d;
                }
            }
            if (it == 0) TRACE(21);
            if (it == nw) TRACE(22);
        }
    }
    __syncthreads();
    TRACE(11);
    // ---- weighted sum in top-k order, + shared (moe_layer.py:85-86, 102-105)
    for (int rr = tid; rr < nh; rr += kFusedThreads) {
        float comb = 0.f;
        int a = 0;
        for (int k = 0; k < K; ++k) {
            if (a < A && s_act[a] == k) {
                comb = __fadd_rn(comb, __fmul_rn(s_w[k], s_vout[a * p.max_out_rows + rr]));
                ++a;
            }
        }
        if (Is) comb = __fadd_rn(comb, __fmul_rn(*s_sg, s_vout[A * p.max_out_rows + rr]));
        p.y[h0 + rr] = comb;
    }
    // ---- exit: the last CTA resets the counters for the next launch
    __syncthreads();
    TRACE(12);
#undef TRACE
    if (tid == 0) {
        __threadfence();
        const uint32_t t = atomicAdd(p.ctr + C_EXIT, 1u);
        if (t == (uint32_t)G - 1) {
            p.ctr[C_ROUTER] = 0;
            p.ctr[C_SHARED] = 0;
            p.ctr[C_GATEUP] = 0;
            p.ctr[C_EXIT] = 0;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ host side

static inline uint32_t a16(uint32_t v) { return (v + 127) & ~127u; }

static int lanes_per_row(int cols) {
    const int pairs = cols / 64;
    return pairs;  // 4, 8, 16 or 32 (checked by fused_plan)
}

bool fused_supported(const moe_b200_layer* L, int T, int flags) {
    if (T != 1 || (flags & (MOE_B200_EXACT | MOE_B200_FP16_GRAPH | MOE_B200_SHARED_ONLY))) return false;
    auto ok_cols = [](int cols) {
        if (cols % 256) return false;
        const int pairs = cols / 64;
        return pairs == 4 || pairs == 8 || pairs == 16 || pairs == 32;
    };
    if (!ok_cols(L->hidden) || !ok_cols(L->intermediate)) return false;
    if (L->top_k > kMaxTopK) return false;
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    if (shared && !ok_cols(L->shared_intermediate)) return false;
    auto rb16 = [](int t, int cols) { return row_bytes(t, cols) % 16 == 0; };
    if (!rb16(L->gate_type, L->hidden) || !rb16(L->up_type, L->hidden) ||
        !rb16(L->down_type, L->intermediate))
        return false;
    if (shared && (!rb16(L->shared_gate_type, L->hidden) || !rb16(L->shared_up_type, L->hidden) ||
                   !rb16(L->shared_down_type, L->shared_intermediate)))
        return false;
    return true;
}

size_t fused_workspace_bytes(const moe_b200_layer* L) {
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate : L->intermediate;
    return 256 + align_up((size_t)L->n_experts * 4) + align_up((size_t)L->top_k * L->intermediate * 4) +
           align_up((size_t)Imax * 4) + 256;
}

static bool fused_plan(const moe_b200_layer* L, bool shared, int G, FusedParams& p) {
    const int H = L->hidden, I = L->intermediate, E = L->n_experts, K = L->top_k;
    const int Is = shared ? L->shared_intermediate : 0;
    const int Imax = Is > I ? Is : I;
    p.G = G;
    p.with_shared = shared ? 1 : 0;
    p.max_router_rows = (E + G - 1) / G;
    p.max_sgu_rows = Is ? (Is + G - 1) / G : 0;
    p.max_out_rows = (H + G - 1) / G;
    p.max_rgu_rows = (K * I + G - 1) / G;
    p.lpr_h = lanes_per_row(H);
    p.lpr_i = lanes_per_row(I);
    p.lpr_is = Is ? lanes_per_row(Is) : 4;
    // chunks of a multiple of 16 rows, at most kMaxChunks of them
    p.chunk_rows = 16 * ((p.max_rgu_rows + 16 * kMaxChunks - 1) / (16 * kMaxChunks));
    uint32_t o = 0;
    auto take = [&](uint64_t bytes) {
        const uint32_t at = o;
        o = a16(o + (uint32_t)bytes);
        return at;
    };
    p.o_x32 = take((uint64_t)H * 4);
    p.o_xq = take(qvec_bytes(H));
    p.o_router = take((uint64_t)p.max_router_rows * H * 4);
    p.o_sgate = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_gate_type, H) : 0);
    p.o_sup = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_up_type, H) : 0);
    p.o_sdown = take(Is ? (uint64_t)p.max_out_rows * row_bytes(L->shared_down_type, Is) : 0);
    p.o_rgate = take((uint64_t)p.max_rgu_rows * row_bytes(L->gate_type, H));
    p.o_rup = take((uint64_t)p.max_rgu_rows * row_bytes(L->up_type, H));
    p.o_rdown = take((uint64_t)K * p.max_out_rows * row_bytes(L->down_type, I));
    p.o_act = take((uint64_t)(K + 1) * Imax * 4);
    p.o_aq = take((uint64_t)(K + 1) * qvec_bytes(Imax));
    p.o_misc = take(512 + ((5 * E + 15) & ~15) + (uint64_t)(K + 1) * p.max_out_rows * 4);
    p.total = o;
    return p.total <= 227 * 1024;
}

static thread_local uint64_t* tl_trace = nullptr;
static thread_local int tl_trace_cap = 0;

void set_fused_trace(void* buf, int capacity_ctas) {
    tl_trace = static_cast<uint64_t*>(buf);
    tl_trace_cap = capacity_ctas;
}

uint64_t* trace_buffer(int* capacity_ctas) {
    *capacity_ctas = tl_trace_cap;
    return tl_trace;
}

cudaError_t launch_decode_fused(const moe_b200_layer* L, int flags, const float* x, float* y,
                                int32_t* ids_out, float* w_out, void* ws, cudaStream_t stream,
                                bool* launched) {
    *launched = false;
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    FusedParams p{};
    p.L = *L;
    const int G = sm_count();
    if (!fused_plan(L, shared, G, p)) return cudaSuccess;
    using KernelFn = void (*)(FusedParams);
    struct Instance {
        int gu, dn, sgu, sdn;
        KernelFn fn;
    };
    static const Instance kInstances[] = {
        {Q3_K, Q4_K, Q8_0, Q8_0, k_decode_fused<Q3_K, Q4_K, Q8_0, Q8_0>},
        {Q4_K, Q4_K, Q8_0, Q8_0, k_decode_fused<Q4_K, Q4_K, Q8_0, Q8_0>},
        {Q4_K, Q8_0, Q8_0, Q8_0, k_decode_fused<Q4_K, Q8_0, Q8_0, Q8_0>},
        {Q3_K, Q8_0, Q8_0, Q8_0, k_decode_fused<Q3_K, Q8_0, Q8_0, Q8_0>},
        {-1, -1, -1, -1, k_decode_fused<-1, -1, -1, -1>},
    };
    constexpr int kNumInstances = sizeof(kInstances) / sizeof(kInstances[0]);
    int pick = kNumInstances - 1;
    for (int i = 0; i + 1 < kNumInstances; ++i) {
        const Instance& in = kInstances[i];
        const bool gu = L->gate_type == in.gu && L->up_type == in.gu && L->down_type == in.dn;
        const bool sh = !shared || (L->shared_gate_type == in.sgu && L->shared_up_type == in.sgu &&
                                    L->shared_down_type == in.sdn);
        if (gu && sh) {
            pick = i;
            break;
        }
    }
    static bool attr_set[64][8] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev][pick]) {
        cudaError_t e = cudaFuncSetAttribute(kInstances[pick].fn,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        attr_set[dev][pick] = true;
    }
    char* base = static_cast<char*>(ws);
    p.x = x;
    p.y = y;
    p.ids_out = ids_out;
    p.w_out = w_out;
    p.ctr = reinterpret_cast<uint32_t*>(base);
    size_t off = 256;
    p.scores = reinterpret_cast<float*>(base + off);
    off += align_up((size_t)L->n_experts * 4);
    p.act_r = reinterpret_cast<float*>(base + off);
    off += align_up((size_t)L->top_k * L->intermediate * 4);
    p.act_s = reinterpret_cast<float*>(base + off);
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate : L->intermediate;
    off += align_up((size_t)Imax * 4);
    p.sg = reinterpret_cast<float*>(base + off);
    p.trace = (tl_trace && tl_trace_cap >= G) ? tl_trace : nullptr;
    static const bool no_warm = getenv("MOE_B200_NO_WARM") != nullptr;
    p.warm = no_warm ? 0 : 1;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = p.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, kInstances[pick].fn, p);
    if (e == cudaSuccess) *launched = true;
    return e;
}

}  // namespace moeb200
