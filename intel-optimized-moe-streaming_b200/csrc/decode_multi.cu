// decode_multi.cu -- fused layer decode of up to 8 tokens in one cooperative
// launch (batched decode, and the expert-parallel step in which every rank
// runs all gathered tokens through the experts it holds).
//
// Same layer as the single-token kernel (reference run_moe_layer,
// src/flash_moe/moe_layer.py:39-107, with moe_quant_expert,
// cpp/moe_quant_dot.cpp:171-214, per selected expert), for T tokens:
//
//   router rows [E*c/G, E*(c+1)/G) of CTA c, dotted with every token;
//   top-k of token t by warp t (every CTA, identically, from the E x T
//     scores in the workspace);
//   "pairs": the (token, slot) selections whose expert this GPU holds,
//     token-major, P <= T*K of them; routed gate/up work is the flattened
//     (pair, row) range [P*I*c/G, P*I*(c+1)/G) of CTA c, so every CTA does
//     ~1/G of the dot products whatever the routing (a row of an expert two
//     tokens share is fetched twice, the second time from L2);
//   down rows [H*c/G, H*(c+1)/G) of every pair and of the shared expert;
//   weighted sum in top-k order + sigmoid-gated shared expert per token.
//
// Weight rows stream through a ring of shared-memory slots filled by TMA
// bulk copies (no multicast): the routed gate/up rows of the CTA's range in
// chunks, then the down rows of the pairs.  All chunks that fit are issued as
// soon as the routing is known; a slot is refilled after a CTA barrier once
// every warp is done with it.  The shared expert's rows are copied at kernel
// entry and stay resident.  Two grid-wide phases (router -> top-k, gate/up
// -> down) synchronise through release/acquire counters in the workspace
// with bounded waits (a wait that gives up records -9 in the error word).
//
// The shared expert is added to tokens [sh_lo, sh_hi) only: the whole batch
// in a plain batched call; one rank's own tokens in the expert-parallel step
// (the other ranks' partial outputs then carry routed experts only, and the
// sum over ranks counts the shared expert once).
#include <math.h>
#include <string.h>

#include <new>

#include "fused.cuh"
#include "launch.h"
#include "qdot.cuh"
#include "sm100.cuh"
#include "topk.cuh"

namespace moeb200 {

constexpr int kMultiMaxTokens = 8;
constexpr int kRing = 4;  // ring slots
constexpr int kBarRouter = 0, kBarShared = 1, kBarX = 2, kBarRing = 3;
constexpr int kMultiMisc = 2560;  // barriers + routing tables (offsets below)

// Expert-parallel exchange over peer memory: every rank has one exchange
// buffer, mapped into every other rank's address space, of exchange words
// (payload + step number in one 64-bit store, see st_word_sys):
//   xs    [world*tq][H]    gathered tokens (rank r's rows r*tq..)
//   yp    [world][tq][H]   partial outputs of this rank's tokens, by sender
//   seq                    steps run (this rank's copy only)
struct EpView {
    int world, rank, tq;
    const float* x_own;          // [tq][H] this rank's tokens
    float* y_own;                // [tq][H] their layer outputs
    const uint64_t* xs;          // local buffer
    const uint64_t* yp;
    uint32_t* seq;
    uint64_t* xs_peer[kMultiMaxTokens];    // the same regions of rank q (q = rank: local)
    uint64_t* yp_peer[kMultiMaxTokens];
};

struct MultiParams {
    moe_b200_layer L;
    const float* x;      // [T][H]
    float* y;            // [T][H]
    int32_t* ids_out;    // [T][K] or null
    float* w_out;        // [T][K] or null
    int T;
    int routed;          // 0: shared expert only (no router, no routed experts)
    int sh_lo, sh_hi;    // tokens given the shared expert
    uint32_t* ctr;       // counters, error word at ctr[C_ERROR]
    float* scores;       // [T][E]
    float* act_r;        // [T*K][I]   pair-major routed activations
    float* act_s;        // [T][Is]    shared activations (token index)
    float* sg;           // [T]        shared gate (token index)
    int G;
    int max_router_rows, max_sgu_rows, max_out_rows;
    int lpr_h, lpr_i, lpr_is;
    int slot_bytes;      // ring slot size
    int gu_rows;         // routed gate/up rows that fit one slot
    int dn_pairs;        // pairs whose down rows [h0, h1) fit one slot
    uint32_t o_vout, o_sgate, o_sup, o_sdown, o_q, o_ring, total;
    uint64_t* trace;     // [G x 32] phase timestamps (ns), or null
    EpView ep;           // peer-memory exchange (ep.world > 0), else unused
};

template <int GU, int DN, int SGU, int SDN>
__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_multi(const __grid_constant__ MultiParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const moe_b200_layer& L = p.L;
    const int c = blockIdx.x, G = p.G, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int nw = kFusedThreads / 32;
    const int T = p.T, H = L.hidden, I = L.intermediate, E = L.n_experts, K = L.top_k;
    const int TK = T * K;
    const int ns = p.sh_hi - p.sh_lo;
    const int Is = ns > 0 ? L.shared_intermediate : 0;
    const int ebeg = L.expert_begin, ecnt = L.expert_count;
    const int64_t rb_gate = row_bytes(L.gate_type, H), rb_up = row_bytes(L.up_type, H);
    const int64_t rb_down = row_bytes(L.down_type, I);
    const int64_t st_gate = rb_gate * I, st_up = rb_up * I, st_down = rb_down * H;
    const int64_t rb_sg = Is ? row_bytes(L.shared_gate_type, H) : 0;
    const int64_t rb_su = Is ? row_bytes(L.shared_up_type, H) : 0;
    const int64_t rb_sd = Is ? row_bytes(L.shared_down_type, Is) : 0;
    const int Imax = max(I, Is);

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm);            // [kBarRing + kRing]
    int* s_ids = reinterpret_cast<int*>(sm + 128);               // [TK] selected experts
    float* s_w = reinterpret_cast<float*>(sm + 640);             // [TK] routing weights
    int* s_pt = reinterpret_cast<int*>(sm + 1152);               // [P] pair -> t*K + k
    int* s_tp = reinterpret_cast<int*>(sm + 1664);               // [TK] t*K + k -> pair or -1
    int* s_np = reinterpret_cast<int*>(sm + 2176);
    float* s_sg = reinterpret_cast<float*>(sm + 2192);           // [kMultiMaxTokens]
    float* s_vout = reinterpret_cast<float*>(sm + p.o_vout);     // [TK + T][max_out_rows]
    uint8_t* qbase = sm + p.o_q;   // token codes (gate/up), then activation codes (down)
    float* x32 = reinterpret_cast<float*>(sm + p.o_ring);       // [T][H] until the routing
    float* router_s = x32 + (size_t)T * H;                       // router rows until the routing
    const uint32_t qbH = qvec_bytes(H), qbI = qvec_bytes(Imax);
    const int MO = p.max_out_rows;

    const int r0 = part(E, c, G), r1 = part(E, c + 1, G);
    const int s0 = part(Is, c, G), s1 = part(Is, c + 1, G);
    const int h0 = part(H, c, G), h1 = part(H, c + 1, G);
    const int nh = h1 - h0;
    const int lpr_h = p.lpr_h, sub_h = lane / lpr_h, pr_h = lane % lpr_h;

    if (tid == 0) {
        for (int i = 0; i < kBarRing + kRing; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    uint64_t* trace = p.trace ? p.trace + (size_t)c * kTraceSlots : nullptr;
#define TRACE(i) do { if (trace && tid == 0) trace[i] = global_ns(); } while (0)
    TRACE(0);
    const EpView& ep = p.ep;
    const bool xch = ep.world > 0;
    const uint32_t seq = xch ? *reinterpret_cast<volatile uint32_t*>(ep.seq) + 1u : 0u;
    if (tid == 0) {
        if (!xch) {
            mbar_arrive_expect_tx(&bars[kBarX], (uint32_t)(T * H * 4));
            bulk_g2s(x32, p.x, (uint32_t)(T * H * 4), &bars[kBarX]);
        }
        if (p.routed) {
            mbar_arrive_expect_tx(&bars[kBarRouter], (uint32_t)((r1 - r0) * H * 4));
            if (r1 > r0)
                bulk_g2s(router_s, L.router + (size_t)r0 * H, (uint32_t)((r1 - r0) * H * 4),
                         &bars[kBarRouter]);
        }
        if (Is) {
            mbar_arrive_expect_tx(&bars[kBarShared],
                                  (uint32_t)((s1 - s0) * (rb_sg + rb_su) + nh * rb_sd));
            if (s1 > s0) {
                bulk_g2s(sm + p.o_sgate, L.shared_gate + s0 * rb_sg, (uint32_t)((s1 - s0) * rb_sg),
                         &bars[kBarShared]);
                bulk_g2s(sm + p.o_sup, L.shared_up + s0 * rb_su, (uint32_t)((s1 - s0) * rb_su),
                         &bars[kBarShared]);
            }
            if (nh > 0)
                bulk_g2s(sm + p.o_sdown, L.shared_down + h0 * rb_sd, (uint32_t)(nh * rb_sd),
                         &bars[kBarShared]);
        }
    }

    // ---- the tokens; router scores of rows [r0, r1), one warp per (row, token)
    if (xch) {
        // dispatch: CTA q < world writes this rank's tokens into rank q's
        // gathered-token rows; every CTA then reads all ranks' tokens from
        // its own buffer as their words arrive
        if (c < ep.world) {
            uint64_t* dst = ep.xs_peer[c] + (size_t)ep.rank * ep.tq * H;
            for (int i = tid; i < ep.tq * H; i += kFusedThreads) st_word_sys(dst + i, ep.x_own[i], seq);
            TRACE(1);
        }
        // word pairs pi = tid + u * kFusedThreads, all kXPairs of a thread's
        // round in flight (one poll round trip for all of them, not one per
        // word); only the pairs still missing are read again
        constexpr int kXPairs = 8;
        bool ok = true;
        const int n_pairs = T * H / 2;
        for (int p0 = tid; p0 < n_pairs && ok; p0 += kXPairs * kFusedThreads) {
            uint32_t pend = 0;
#pragma unroll
            for (int u = 0; u < kXPairs; ++u)
                if (p0 + u * kFusedThreads < n_pairs) pend |= 1u << u;
            for (uint32_t round = 0; pend != 0u; ++round) {
                if (round == kWaitPolls) {
                    ok = false;
                    break;
                }
                ulonglong2 wv[kXPairs];
#pragma unroll
                for (int u = 0; u < kXPairs; ++u)
                    wv[u] = ((pend >> u) & 1u) ? ld_word2_sys(ep.xs + 2 * (p0 + u * kFusedThreads))
                                               : make_ulonglong2(0ull, 0ull);
#pragma unroll
                for (int u = 0; u < kXPairs; ++u)
                    if (((pend >> u) & 1u) && (uint32_t)(wv[u].x >> 32) == seq &&
                        (uint32_t)(wv[u].y >> 32) == seq) {
                        pend &= ~(1u << u);
                        *reinterpret_cast<float2*>(x32 + 2 * (p0 + u * kFusedThreads)) =
                            make_float2(__uint_as_float((uint32_t)wv[u].x), __uint_as_float((uint32_t)wv[u].y));
                    }
            }
        }
        if (!ok) set_error(p.ctr, ST_TIMEOUT);
    } else if (tid == 0 && !mbar_wait(&bars[kBarX], 0, kWaitPolls)) {
        set_error(p.ctr, ST_TIMEOUT);
    }
    if (p.routed && tid == 0 && !mbar_wait(&bars[kBarRouter], 0, kWaitPolls))
        set_error(p.ctr, ST_TIMEOUT);
    __syncthreads();
    TRACE(2);
    if (p.routed) {
        const float* bias = L.router_bias;
        const int R = r1 - r0;
        for (int it = warp; it < R * T; it += nw) {
            const int rr = it / T, t = it % T;
            float acc = dot_f32_warp(router_s + (size_t)rr * H, x32 + (size_t)t * H, H, lane);
            if (lane == 0) {
                if (bias) acc = __fadd_rn(acc, bias[r0 + rr]);
                p.scores[(size_t)t * E + r0 + rr] = acc;
            }
        }
        __syncthreads();
        if (tid == 0) red_release_add(p.ctr + C_ROUTER, 1);
        TRACE(3);
    }

    // ---- token codes for the integer dot products; shared gates (CTA 0)
    for (int it = warp; it < T * (H / 256); it += nw) {
        const int t = it / (H / 256), b = it % (H / 256);
        quantize_block_warp(x32 + (size_t)t * H, qvec_at(qbase + t * qbH, H), b);
    }
    if (Is && c == 0) {
        const float* ginp = L.shared_gate_inp;
        for (int j = nw - 1 - warp; j < ns; j += nw) {
            const float* xt = x32 + (size_t)(p.sh_lo + j) * H;
            float acc = 0.f;
            for (int i = lane; i < H; i += 32) acc = fmaf(xt[i], ginp[i], acc);
            acc = warp_sum(acc);
            if (lane == 0) p.sg[p.sh_lo + j] = shared_sigmoid(acc);
        }
    }
    // the ring reuses the token and router region: order these reads before
    // the copies issued after the next barrier
    fence_proxy_async_smem();
    __syncthreads();

    // ---- routing of every token (every CTA, identically) and the pair table
    if (p.routed) {
        if (tid == 0 && !wait_flag(p.ctr + C_ROUTER, (uint32_t)G, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        __syncthreads();
        TRACE(4);
        if (warp < T) topk_softmax_warp_fast(p.scores + (size_t)warp * E, E, K, s_ids + warp * K, s_w + warp * K);
        __syncthreads();
        if (warp == 0) {
            int base = 0;
            for (int j0 = 0; j0 < TK; j0 += 32) {
                const int j = j0 + lane;
                bool held = false;
                if (j < TK) {
                    const int e = s_ids[j];
                    held = e >= ebeg && e < ebeg + ecnt;
                }
                const unsigned m = __ballot_sync(0xffffffffu, held);
                if (held) {
                    const int pi = base + __popc(m & ((1u << lane) - 1u));
                    s_pt[pi] = j;
                    s_tp[j] = pi;
                } else if (j < TK) {
                    s_tp[j] = -1;
                }
                base += __popc(m);
            }
            if (lane == 0) *s_np = base;
        }
        if (c == 0) {
            for (int j = tid; j < TK; j += kFusedThreads) {
                if (p.ids_out) p.ids_out[j] = s_ids[j];
                if (p.w_out) p.w_out[j] = s_w[j];
            }
        }
        __syncthreads();
    }
    const int P = p.routed ? *s_np : 0;
    TRACE(5);

    // ---- ring plan (identical in every thread)
    const int f0 = part(P * I, c, G), f1 = part(P * I, c + 1, G);
    const int nrows = f1 - f0;
    const int n_gu = (nrows + p.gu_rows - 1) / p.gu_rows;
    const int crow = n_gu ? (nrows + n_gu - 1) / n_gu : 0;  // balanced chunk rows
    const int DP = p.dn_pairs;
    const int n_dn = (nh > 0 && P > 0) ? (P + DP - 1) / DP : 0;
    const int NC = n_gu + n_dn;
    auto slot = [&](int q) { return sm + p.o_ring + (size_t)(q % kRing) * p.slot_bytes; };
    auto issue = [&](int q) {
        uint8_t* dst = slot(q);
        uint64_t* bar = &bars[kBarRing + q % kRing];
        if (q < n_gu) {
            const int q0 = q * crow, q1 = min(nrows, q0 + crow);
            mbar_arrive_expect_tx(bar, (uint32_t)((q1 - q0) * (rb_gate + rb_up)));
            for (int f = f0 + q0; f < f0 + q1;) {
                const int pi = f / I, r = f % I;
                const int n = min(f0 + q1 - f, I - r);
                const int64_t e = s_ids[s_pt[pi]] - ebeg;
                const int at = f - f0 - q0;
                bulk_g2s(dst + at * rb_gate, L.gate + e * st_gate + r * rb_gate, (uint32_t)(n * rb_gate), bar);
                bulk_g2s(dst + p.gu_rows * rb_gate + at * rb_up, L.up + e * st_up + r * rb_up,
                         (uint32_t)(n * rb_up), bar);
                f += n;
            }
        } else {
            const int j0 = (q - n_gu) * DP, j1 = min(P, j0 + DP);
            mbar_arrive_expect_tx(bar, (uint32_t)((j1 - j0) * nh * rb_down));
            for (int j = j0; j < j1; ++j) {
                const int64_t e = s_ids[s_pt[j]] - ebeg;
                bulk_g2s(dst + (j - j0) * nh * rb_down, L.down + e * st_down + h0 * rb_down,
                         (uint32_t)(nh * rb_down), bar);
            }
        }
    };
    if (warp == 0 && lane < min(kRing, NC)) issue(lane);
    uint32_t ring_ph = 0;  // parity of each slot's mbarrier phase
    auto wait_slot = [&](int q) {
        const int sl = q % kRing;
        if (!mbar_wait(&bars[kBarRing + sl], (ring_ph >> sl) & 1u, kWaitPolls) && lane == 0)
            set_error(p.ctr, ST_TIMEOUT);
        ring_ph ^= 1u << sl;
    };
    auto refill = [&](int q) {  // after chunk q: its slot takes chunk q + kRing
        if (q + kRing < NC) {
            fence_proxy_async_smem();
            __syncthreads();
            if (tid == 0) issue(q + kRing);
        }
    };

    // ---- shared expert gate/up of tokens [sh_lo, sh_hi) while the routed
    // rows are in flight (warp 0, which issued the copies, comes last)
    if (Is) {
        if (!mbar_wait(&bars[kBarShared], 0, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
        const int nsr = s1 - s0, rpw = 32 / lpr_h;
        int cur = -1;
        XLane xl;
        for (int rb = (nw - 1 - warp) * rpw; rb < ns * nsr; rb += nw * rpw) {
            const int i = rb + sub_h;
            const bool ok = i < ns * nsr;
            const int ii = ok ? i : 0;
            const int t = p.sh_lo + ii / nsr, rr = ii % nsr;
            if (t != cur) {
                load_xlane(xl, qvec_at(qbase + t * qbH, H), pr_h >> 2, pr_h & 3);
                cur = t;
            }
            float g = qdot_t<SGU>(L.shared_gate_type, sm + p.o_sgate + rr * rb_sg, pr_h >> 2, pr_h & 3, xl);
            float u = qdot_t<SGU>(L.shared_up_type, sm + p.o_sup + rr * rb_su, pr_h >> 2, pr_h & 3, xl);
            g = group_sum(g, lpr_h);
            u = group_sum(u, lpr_h);
            if (ok && pr_h == 0) p.act_s[(size_t)t * Is + s0 + rr] = (g * shared_sigmoid(g)) * u;
        }
    }

    TRACE(6);
    // ---- routed gate/up, chunk by chunk
    {
        const int rpw = 32 / lpr_h;
        int cur = -1;
        XLane xl;
        for (int q = 0; q < n_gu; ++q) {
            wait_slot(q);
            const uint8_t* src = slot(q);
            const int q0 = q * crow, n = min(crow, nrows - q0);
            for (int rb = warp * rpw; rb < n; rb += nw * rpw) {
                const int rr = rb + sub_h;
                const bool ok = rr < n;
                const int rs = ok ? rr : 0;
                const int f = f0 + q0 + rs;
                const int t = s_pt[f / I] / K;
                if (t != cur) {
                    load_xlane(xl, qvec_at(qbase + t * qbH, H), pr_h >> 2, pr_h & 3);
                    cur = t;
                }
                float g = qdot_t<GU>(L.gate_type, src + rs * rb_gate, pr_h >> 2, pr_h & 3, xl);
                float u = qdot_t<GU>(L.up_type, src + p.gu_rows * rb_gate + rs * rb_up, pr_h >> 2, pr_h & 3, xl);
                g = group_sum(g, lpr_h);
                u = group_sum(u, lpr_h);
                if (ok && pr_h == 0) {
                    const float sgm = 1.0f / (1.0f + expf(-g));
                    p.act_r[f] = (g * sgm) * u;
                }
            }
            refill(q);
        }
    }
    __syncthreads();
    TRACE(7);
    if (tid == 0) {
        red_release_add(p.ctr + C_GATEUP, 1);
        if (!wait_flag(p.ctr + C_GATEUP, (uint32_t)G, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
    }
    __syncthreads();
    TRACE(8);

    // ---- activation codes: pair v < P (routed), P + j (shared of token sh_lo + j)
    {
        const int bi = I / 256, bs = Is / 256;
        for (int it = warp; it < P * bi + ns * bs; it += nw) {
            if (it < P * bi) {
                const int v = it / bi, b = it % bi;
                quantize_block_gmem(p.act_r + (size_t)v * I, qvec_at(qbase + v * qbI, I), b);
            } else {
                const int j = (it - P * bi) / bs, b = (it - P * bi) % bs;
                quantize_block_gmem(p.act_s + (size_t)(p.sh_lo + j) * Is,
                                    qvec_at(qbase + (P + j) * qbI, Is), b);
            }
        }
        if (tid < ns) s_sg[tid] = __ldcg(p.sg + p.sh_lo + tid);
    }
    __syncthreads();
    TRACE(9);

    // ---- down rows [h0, h1): item = (vector, pair of row groups)
    if (Is) {
        const int lpr = p.lpr_is, rpw = 32 / lpr, sub = lane / lpr, pr = lane % lpr;
        const int ng = (nh + rpw - 1) / rpw, np = (ng + 1) / 2;
        for (int it = warp; it < ns * np; it += nw) {
            const int j = it / np, gp = it % np;
            XLane xa;
            load_xlane(xa, qvec_at(qbase + (P + j) * qbI, Is), pr >> 2, pr & 3);
#pragma unroll
            for (int gg = 0; gg < 2; ++gg) {
                const int gi = 2 * gp + gg;
                if (gi < ng) {
                    const int rr = gi * rpw + sub;
                    const bool ok = rr < nh;
                    float d = qdot_t<SDN>(L.shared_down_type, sm + p.o_sdown + (ok ? rr : 0) * rb_sd,
                                          pr >> 2, pr & 3, xa);
                    d = group_sum(d, lpr);
                    if (ok && pr == 0) s_vout[(TK + j) * MO + rr] = d;
                }
            }
        }
    }
    {
        const int lpr = p.lpr_i, rpw = 32 / lpr, sub = lane / lpr, pr = lane % lpr;
        const int ng = (nh + rpw - 1) / rpw, np = (ng + 1) / 2;
        for (int q = n_gu; q < NC; ++q) {
            wait_slot(q);
            const uint8_t* src = slot(q);
            const int j0 = (q - n_gu) * DP, j1 = min(P, j0 + DP);
            for (int it = warp; it < (j1 - j0) * np; it += nw) {
                const int j = j0 + it / np, gp = it % np;
                XLane xa;
                load_xlane(xa, qvec_at(qbase + j * qbI, I), pr >> 2, pr & 3);
                const uint8_t* rows = src + (int64_t)(j - j0) * nh * rb_down;
#pragma unroll
                for (int gg = 0; gg < 2; ++gg) {
                    const int gi = 2 * gp + gg;
                    if (gi < ng) {
                        const int rr = gi * rpw + sub;
                        const bool ok = rr < nh;
                        float d = qdot_t<DN>(L.down_type, rows + (ok ? rr : 0) * rb_down, pr >> 2, pr & 3, xa);
                        d = group_sum(d, lpr);
                        if (ok && pr == 0) s_vout[j * MO + rr] = d;
                    }
                }
            }
            refill(q);
        }
    }
    __syncthreads();
    TRACE(10);

    // ---- weighted sum in top-k order, + shared (moe_layer.py:85-86, 102-105)
    for (int i = tid; i < T * nh; i += kFusedThreads) {
        const int t = i / nh, rr = i % nh;
        float comb = 0.f;
        if (p.routed) {
            for (int k = 0; k < K; ++k) {
                const int pi = s_tp[t * K + k];
                if (pi >= 0) comb = __fadd_rn(comb, __fmul_rn(s_w[t * K + k], s_vout[pi * MO + rr]));
            }
        }
        if (t >= p.sh_lo && t < p.sh_hi)
            comb = __fadd_rn(comb, __fmul_rn(s_sg[t - p.sh_lo], s_vout[(TK + t - p.sh_lo) * MO + rr]));
        if (xch) {
            // combine: the partial row goes to the token's owner
            const int q = t / ep.tq, j = t % ep.tq;
            st_word_sys(ep.yp_peer[q] + ((size_t)ep.rank * ep.tq + j) * H + h0 + rr, comb, seq);
        } else {
            p.y[(size_t)t * H + h0 + rr] = comb;
        }
    }
    if (xch) {
        // CTA c of every rank sends rows [h0, h1) of its partials; the own
        // tokens' rows are the sum over ranks in rank order
        TRACE(11);
        // every (rank, own token, row) word polled at once into shared
        // memory (the partial-output rows are free: the loop above has read
        // them), then each own row summed over the ranks in rank order
        __syncthreads();
        float* s_comb = s_vout;  // [world][tq * nh]
        const int per = ep.tq * nh, n_words = ep.world * per;
        bool ok = true;
        for (int i0 = tid; i0 < n_words && ok; i0 += 4 * kFusedThreads) {
            uint32_t pend = 0;
            const uint64_t* src[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const int i = i0 + u * kFusedThreads;
                if (i < n_words) pend |= 1u << u;
                const int r = i / per, rem = i - r * per, j = rem / nh, rr = rem - j * nh;
                src[u] = ep.yp + ((size_t)r * ep.tq + j) * H + h0 + rr;
            }
            for (uint32_t round = 0; pend != 0u; ++round) {
                if (round == kWaitPolls) {
                    ok = false;
                    break;
                }
                uint64_t wv[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) wv[u] = ((pend >> u) & 1u) ? ld_word_sys(src[u]) : 0ull;
#pragma unroll
                for (int u = 0; u < 4; ++u)
                    if (((pend >> u) & 1u) && (uint32_t)(wv[u] >> 32) == seq) {
                        pend &= ~(1u << u);
                        s_comb[i0 + u * kFusedThreads] = __uint_as_float((uint32_t)wv[u]);
                    }
            }
        }
        if (!ok) set_error(p.ctr, ST_TIMEOUT);
        __syncthreads();
        for (int i = tid; i < per; i += kFusedThreads) {
            const int j = i / nh, rr = i - j * nh;
            float acc = 0.f;
            for (int r = 0; r < ep.world; ++r) acc = __fadd_rn(acc, s_comb[r * per + i]);
            ep.y_own[(size_t)j * H + h0 + rr] = acc;
        }
        TRACE(12);
    }

    TRACE(13);
#undef TRACE
    // ---- exit: the last CTA resets the counters for the next launch
    if (tid == 0) {
        __threadfence();
        const uint32_t t = atomicAdd(p.ctr + C_EXIT, 1u);
        if (t == (uint32_t)G - 1) {
            p.ctr[C_ROUTER] = 0;
            p.ctr[C_GATEUP] = 0;
            p.ctr[C_EXIT] = 0;
            if (xch) *ep.seq = seq;
            __threadfence();
        }
    }
}

// ------------------------------------------------------------------ host side

static inline uint32_t a128(uint32_t v) { return (v + 127) & ~127u; }

static bool ok_cols(int cols) {
    if (cols % 256) return false;
    const int pairs = cols / 64;
    return pairs == 4 || pairs == 8 || pairs == 16 || pairs == 32;
}

static bool multi_plan(const moe_b200_layer* L, int T, bool routed, int ns, int G, MultiParams& p) {
    const int H = L->hidden, I = L->intermediate, E = L->n_experts, K = L->top_k;
    const int Is = ns > 0 ? L->shared_intermediate : 0;
    const int Imax = Is > I ? Is : I;
    const int TK = T * K;
    p.G = G;
    p.max_router_rows = routed ? (E + G - 1) / G : 0;
    p.max_sgu_rows = Is ? (Is + G - 1) / G : 0;
    p.max_out_rows = (H + G - 1) / G;
    p.lpr_h = H / 64;
    p.lpr_i = I / 64;
    p.lpr_is = Is ? Is / 64 : 4;
    uint32_t o = kMultiMisc;
    auto take = [&](uint64_t bytes) {
        const uint32_t at = o;
        o = a128(o + (uint32_t)bytes);
        return at;
    };
    p.o_vout = take((uint64_t)(TK + T) * p.max_out_rows * 4);
    p.o_sgate = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_gate_type, H) : 0);
    p.o_sup = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_up_type, H) : 0);
    p.o_sdown = take(Is ? (uint64_t)p.max_out_rows * row_bytes(L->shared_down_type, Is) : 0);
    const uint64_t qx = (uint64_t)T * qvec_bytes(H), qa = (uint64_t)(TK + T) * qvec_bytes(Imax);
    p.o_q = take(qx > qa ? qx : qa);
    p.o_ring = o;
    const uint32_t limit = 227 * 1024;
    if (o >= limit) return false;
    const uint32_t slot = ((limit - o) / kRing) & ~127u;
    const uint64_t phase_a = (uint64_t)T * H * 4 + (uint64_t)p.max_router_rows * H * 4;
    if ((uint64_t)slot * kRing < phase_a) return false;
    const int64_t gu_pair = row_bytes(L->gate_type, H) + row_bytes(L->up_type, H);
    const int64_t dn_pair = (int64_t)p.max_out_rows * row_bytes(L->down_type, I);
    p.slot_bytes = (int)slot;
    p.gu_rows = (int)(slot / gu_pair);
    p.dn_pairs = (int)(slot / dn_pair);
    if (p.gu_rows < 1 || p.dn_pairs < 1) return false;
    p.total = o + kRing * slot;
    return p.total <= limit;
}

bool multi_supported(const moe_b200_layer* L, int T, int flags) {
    if (T < 1 || T > kMultiMaxTokens) return false;
    if (flags & (MOE_B200_EXACT | MOE_B200_FP16_GRAPH)) return false;
    if (!ok_cols(L->hidden) || !ok_cols(L->intermediate)) return false;
    if (L->top_k > kMaxTopK || L->n_experts > 256) return false;
    const bool shared_only = (flags & MOE_B200_SHARED_ONLY) != 0;
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    if (shared_only && !shared) return false;
    if (shared && !ok_cols(L->shared_intermediate)) return false;
    auto rb16 = [](int t, int cols) { return row_bytes(t, cols) % 16 == 0; };
    if (!rb16(L->gate_type, L->hidden) || !rb16(L->up_type, L->hidden) ||
        !rb16(L->down_type, L->intermediate))
        return false;
    if (shared && (!rb16(L->shared_gate_type, L->hidden) || !rb16(L->shared_up_type, L->hidden) ||
                   !rb16(L->shared_down_type, L->shared_intermediate)))
        return false;
    MultiParams p{};
    return multi_plan(L, T, !shared_only, shared ? T : 0, sm_count(), p);
}

size_t multi_workspace_bytes(const moe_b200_layer* L, int T) {
    const int Is = L->shared_intermediate;
    // counters, scores [T][E], pair activations [T*K][I], shared activations
    // [T][Is], shared gates [T]
    return 256 + align_up((size_t)T * L->n_experts * 4) +
           align_up((size_t)T * L->top_k * L->intermediate * 4) + align_up((size_t)T * Is * 4) +
           align_up((size_t)T * 4);
}

cudaError_t launch_decode_multi(const moe_b200_layer* L, int flags, const float* x, int T,
                                int sh_lo, int sh_hi, float* y, int32_t* ids_out, float* w_out,
                                void* ws, cudaStream_t stream, bool* launched,
                                const moe_b200_ep* xc) {
    *launched = false;
    if (xc) {
        // the exchange fixes the token set and the shared expert's tokens
        if (!xc->connected || T != xc->world * xc->tq || sm_count() != xc->G) return cudaSuccess;
        sh_lo = xc->rank * xc->tq;
        sh_hi = sh_lo + xc->tq;
    }
    const bool shared_only = (flags & MOE_B200_SHARED_ONLY) != 0;
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    if (!shared) sh_lo = sh_hi = 0;
    MultiParams p{};
    p.L = *L;
    const int G = sm_count();
    if (!multi_plan(L, T, !shared_only, sh_hi - sh_lo, G, p)) return cudaSuccess;
    using KernelFn = void (*)(MultiParams);
    struct Instance {
        int gu, dn, sgu, sdn;
        KernelFn fn;
    };
    static const Instance kInstances[] = {
        {Q3_K, Q4_K, Q8_0, Q8_0, k_decode_multi<Q3_K, Q4_K, Q8_0, Q8_0>},
        {Q4_K, Q4_K, Q8_0, Q8_0, k_decode_multi<Q4_K, Q4_K, Q8_0, Q8_0>},
        {-1, -1, -1, -1, k_decode_multi<-1, -1, -1, -1>},
    };
    constexpr int kNumInstances = sizeof(kInstances) / sizeof(kInstances[0]);
    int pick = kNumInstances - 1;
    for (int i = 0; i + 1 < kNumInstances; ++i) {
        const Instance& in = kInstances[i];
        const bool gu = L->gate_type == in.gu && L->up_type == in.gu && L->down_type == in.dn;
        const bool sh = sh_hi == sh_lo || (L->shared_gate_type == in.sgu && L->shared_up_type == in.sgu &&
                                           L->shared_down_type == in.sdn);
        if (gu && sh) {
            pick = i;
            break;
        }
    }
    static bool attr_set[64][4] = {};
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
    if (xc) {
        EpView& v = p.ep;
        v.world = xc->world;
        v.rank = xc->rank;
        v.tq = xc->tq;
        v.x_own = x;
        v.y_own = y;
        for (int q = 0; q < xc->world; ++q) {
            char* b = xc->peer[q];
            v.xs_peer[q] = reinterpret_cast<uint64_t*>(b + xc->o_xs);
            v.yp_peer[q] = reinterpret_cast<uint64_t*>(b + xc->o_yp);
        }
        v.xs = v.xs_peer[xc->rank];
        v.yp = v.yp_peer[xc->rank];
        v.seq = reinterpret_cast<uint32_t*>(xc->local + xc->o_seq);
        p.x = nullptr;
        p.y = nullptr;
    }
    int trace_cap = 0;
    uint64_t* tb = trace_buffer(&trace_cap);
    p.trace = (tb && trace_cap >= G) ? tb : nullptr;
    p.T = T;
    p.routed = shared_only ? 0 : 1;
    p.sh_lo = sh_lo;
    p.sh_hi = sh_hi;
    p.ctr = reinterpret_cast<uint32_t*>(base);
    size_t off = 256;
    p.scores = reinterpret_cast<float*>(base + off);
    off += align_up((size_t)T * L->n_experts * 4);
    p.act_r = reinterpret_cast<float*>(base + off);
    off += align_up((size_t)T * L->top_k * L->intermediate * 4);
    p.act_s = reinterpret_cast<float*>(base + off);
    off += align_up((size_t)T * L->shared_intermediate * 4);
    p.sg = reinterpret_cast<float*>(base + off);

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

// ------------------------------------------------------- exchange context

// What one rank publishes to the others: its buffer's IPC handle and the
// shape every rank must agree on.
struct EpBlob {
    cudaIpcMemHandle_t handle;
    int32_t magic, world, rank, tq, H, G;
    uint64_t bytes;
};
static_assert(sizeof(EpBlob) <= MOE_B200_EP_BLOB_BYTES, "exchange blob too large");
constexpr int32_t kEpMagic = 0x4d4f4550;  // "MOEP"

int ep_create(int world, int rank, int tq, int H, moe_b200_ep** out, void* blob_out,
              cudaError_t* ce) {
    *out = nullptr;
    *ce = cudaSuccess;
    if (world < 2 || world > kMultiMaxTokens || rank < 0 || rank >= world || tq < 1 ||
        world * tq > kMultiMaxTokens || H < 256 || H % 256)
        return ST_ARG;
    auto* c = new (std::nothrow) moe_b200_ep();
    if (!c) return ST_INTERNAL;
    c->world = world;
    c->rank = rank;
    c->tq = tq;
    c->H = H;
    c->G = sm_count();
    cudaGetDevice(&c->dev);
    Stager st;
    c->o_xs = st.take((size_t)world * tq * H * 8);
    c->o_yp = st.take((size_t)world * tq * H * 8);
    c->o_seq = st.take(4);
    c->bytes = st.used;
    cudaError_t e = cudaMalloc(&c->local, c->bytes);
    if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    EpBlob b{};
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&b.handle, c->local);
    if (e != cudaSuccess) {
        if (c->local) cudaFree(c->local);
        delete c;
        *ce = e;
        return ST_CUDA;
    }
    b.magic = kEpMagic;
    b.world = world;
    b.rank = rank;
    b.tq = tq;
    b.H = H;
    b.G = c->G;
    b.bytes = c->bytes;
    memset(blob_out, 0, MOE_B200_EP_BLOB_BYTES);
    memcpy(blob_out, &b, sizeof(b));
    for (int q = 0; q < kMultiMaxTokens; ++q) c->peer[q] = nullptr;
    c->peer[rank] = c->local;
    *out = c;
    return ST_OK;
}

int ep_connect(moe_b200_ep* c, const void* blobs, cudaError_t* ce) {
    *ce = cudaSuccess;
    if (!c || !blobs || c->connected) return ST_ARG;
    const uint8_t* raw = static_cast<const uint8_t*>(blobs);
    for (int q = 0; q < c->world; ++q) {
        EpBlob b;
        memcpy(&b, raw + (size_t)q * MOE_B200_EP_BLOB_BYTES, sizeof(b));
        if (b.magic != kEpMagic || b.world != c->world || b.rank != q || b.tq != c->tq ||
            b.H != c->H || b.G != c->G || b.bytes != c->bytes)
            return ST_ARG;
    }
    for (int q = 0; q < c->world; ++q) {
        if (q == c->rank) continue;
        EpBlob b;
        memcpy(&b, raw + (size_t)q * MOE_B200_EP_BLOB_BYTES, sizeof(b));
        void* ptr = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&ptr, b.handle, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int k = 0; k < q; ++k)
                if (k != c->rank && c->peer[k]) {
                    cudaIpcCloseMemHandle(c->peer[k]);
                    c->peer[k] = nullptr;
                }
            *ce = e;
            return ST_CUDA;
        }
        c->peer[q] = static_cast<char*>(ptr);
    }
    c->connected = true;
    return ST_OK;
}

void ep_destroy(moe_b200_ep* c) {
    if (!c) return;
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(c->dev);
    for (int q = 0; q < c->world; ++q)
        if (q != c->rank && c->peer[q]) cudaIpcCloseMemHandle(c->peer[q]);
    if (c->local) cudaFree(c->local);
    cudaSetDevice(cur);
    delete c;
}

}  // namespace moeb200
