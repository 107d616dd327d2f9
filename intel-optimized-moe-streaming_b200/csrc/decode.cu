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
// E scores, the A*I + Is fp32 activations, the shared gate value, each as a
// 64-bit word of the fp32 value and the step's tag written with one store.
// A CTA polls exactly the words it needs until they carry the current tag:
// no release fence, no counter, no separate data read.  This orders the
// phases on its own when every CTA owns a router row (E >= G): a CTA cannot
// reach step s+2, which reuses step s's buffers, before every CTA has
// written its step s+1 scores, i.e. finished step s.  With E < G the
// counters C_ROUTER / C_GATEUP also separate the phases.
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "fused.cuh"
#include "launch.h"
#include "qdot.cuh"
#include "sm100.cuh"
#include "topk.cuh"

namespace moeb200 {

constexpr int kMaxChunks = 8;  // routed gate/up copy chunks (mbarriers 3..10)
constexpr int kXBar = 3 + kMaxChunks;  // mbarrier of the prefetched token
constexpr int kGatherPairs = 8;  // exchange-word pairs a lane has in flight per poll round

struct FusedParams {
    moe_b200_layer L;        // shapes and block formats of every step's layer
    const float* x;          // single-step launch: the token
    float* y;
    int32_t* ids_out;
    float* w_out;
    const moe_b200_layer* layers;  // multi-step launch: layer table (device)
    const moe_b200_step* steps;    // step table (device), or null
    int n_steps;
    float eps;               // RMSNorm epsilon of MOE_B200_STEP_BLOCK steps
    uint32_t* ctr;           // counters, error word at ctr[C_ERROR]
    uint64_t* scores;        // [2][E]       exchange words (buffer = step parity)
    uint64_t* act_r;         // [2][K x I]
    uint64_t* act_s;         // [2][Imax]
    uint64_t* sg;            // [2]
    uint64_t* trace;         // [G x 32] phase timestamps of step n_steps / 2 (ns), or null
    int* err_out;            // null, or a host-visible word that receives (and clears) the
                             // error word at exit
    int G;
    int with_shared;
    int max_router_rows, max_sgu_rows, max_out_rows, max_rgu_rows;
    int lpr_h, lpr_i, lpr_is;
    int chunk_rows;
    uint32_t o_x32, o_h32, o_xq, o_router, o_sgate, o_sup, o_sdown, o_rgate, o_rup, o_rdown;
    uint32_t o_act, o_aq, o_misc, total;
};

// GU: gate and up type, DN: routed down type, SGU: shared gate and up type,
// SDN: shared down type -- each a ggml type id fixed at compile time, or -1
// to dispatch on the layer's runtime types (the generic instance).
template <int GU, int DN, int SGU, int SDN>
__global__ void __launch_bounds__(kFusedThreads, 1) k_decode_fused(const __grid_constant__ FusedParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    const moe_b200_layer& L0 = p.L;
    const int c = blockIdx.x, G = p.G, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nw = kFusedThreads / 32;
    const int H = L0.hidden, I = L0.intermediate, E = L0.n_experts, K = L0.top_k;
    const int Is = p.with_shared ? L0.shared_intermediate : 0;
    const int ebeg = L0.expert_begin, ecnt = L0.expert_count;
    const int64_t rb_gate = row_bytes(L0.gate_type, H), rb_up = row_bytes(L0.up_type, H);
    const int64_t rb_down = row_bytes(L0.down_type, I);
    const int64_t st_gate = rb_gate * I, st_up = rb_up * I, st_down = rb_down * H;
    const int64_t rb_sg = Is ? row_bytes(L0.shared_gate_type, H) : 0;
    const int64_t rb_su = Is ? row_bytes(L0.shared_up_type, H) : 0;
    const int64_t rb_sd = Is ? row_bytes(L0.shared_down_type, Is) : 0;
    const int Imax = max(I, Is);
    const bool tagged = E >= G;
    const uint32_t seq0 = ld_acquire(p.ctr + C_SEQ);

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + p.o_misc);       // [kXBar + 1]
    int* s_ids = reinterpret_cast<int*>(sm + p.o_misc + 128);          // [16]
    float* s_w = reinterpret_cast<float*>(sm + p.o_misc + 192);        // [16]
    int* s_act = reinterpret_cast<int*>(sm + p.o_misc + 256);          // [16] active slots
    int* s_nact = reinterpret_cast<int*>(sm + p.o_misc + 320);
    float* s_sg = reinterpret_cast<float*>(sm + p.o_misc + 324);
    float* s_part = reinterpret_cast<float*>(sm + p.o_misc + 384);     // [32] partial sums
    float* s_scores = reinterpret_cast<float*>(sm + p.o_misc + 512);   // [E]
    unsigned char* s_taken = reinterpret_cast<unsigned char*>(s_scores + E);
    float* s_vout = reinterpret_cast<float*>(sm + p.o_misc + 512 + ((5 * E + 15) & ~15));
    // per activation vector: the tag of the step whose codes it holds
    volatile uint32_t* s_ready = reinterpret_cast<volatile uint32_t*>(
        sm + p.o_misc + 512 + ((5 * E + 15) & ~15) + (K + 1) * p.max_out_rows * 4);
    float* x32 = reinterpret_cast<float*>(sm + p.o_x32);
    float* h32 = reinterpret_cast<float*>(sm + p.o_h32);

    const int r0 = part(E, c, G), r1 = part(E, c + 1, G);
    const int s0 = part(Is, c, G), s1 = part(Is, c + 1, G);
    const int h0 = part(H, c, G), h1 = part(H, c + 1, G);
    const int nh = h1 - h0;
    const int lpr_h = p.lpr_h, sub_h = lane / lpr_h, pr_h = lane % lpr_h;
    const QVec xq = qvec_at(sm + p.o_xq, H);

    auto step_layer = [&](int s) -> const moe_b200_layer* {
        return p.steps ? p.layers + p.steps[s].layer : &p.L;
    };
    // router rows of step s on bars[0], its shared-expert rows on bars[1]
    auto issue_phase0 = [&](const moe_b200_layer* Ls) {
        const float* router = Ls->router;
        mbar_arrive_expect_tx(&bars[0], (uint32_t)((r1 - r0) * H * 4));
        if (r1 > r0)
            bulk_g2s(sm + p.o_router, router + (size_t)r0 * H, (uint32_t)((r1 - r0) * H * 4), &bars[0]);
        if (Is) {
            const uint8_t* sgp = Ls->shared_gate;
            const uint8_t* sup = Ls->shared_up;
            const uint8_t* sdp = Ls->shared_down;
            mbar_arrive_expect_tx(&bars[1], (uint32_t)((s1 - s0) * (rb_sg + rb_su) + nh * rb_sd));
            if (s1 > s0) {
                bulk_g2s(sm + p.o_sgate, sgp + s0 * rb_sg, (uint32_t)((s1 - s0) * rb_sg), &bars[1]);
                bulk_g2s(sm + p.o_sup, sup + s0 * rb_su, (uint32_t)((s1 - s0) * rb_su), &bars[1]);
            }
            if (nh > 0)
                bulk_g2s(sm + p.o_sdown, sdp + h0 * rb_sd, (uint32_t)(nh * rb_sd), &bars[1]);
        }
    };

    // A step's token comes by TMA (issued before the step begins) unless it
    // is the previous step's output or not 16-byte aligned.
    auto step_x = [&](int s) -> const float* { return p.steps ? p.steps[s].x : p.x; };
    auto x_by_copy = [&](int s) -> bool {
        const bool chain = p.steps && (p.steps[s].flags & MOE_B200_STEP_CHAIN) && s > 0;
        return !chain && (((uintptr_t)step_x(s)) & 15u) == 0;
    };
    auto issue_x = [&](int s) {
        mbar_arrive_expect_tx(&bars[kXBar], (uint32_t)(H * 4));
        bulk_g2s(x32, step_x(s), (uint32_t)(H * 4), &bars[kXBar]);
    };

    if (tid == 0) {
        for (int i = 0; i <= kXBar; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    if (tid <= kMaxTopK) s_ready[tid] = 0u;
    __syncthreads();
    if (tid == 0) {
        issue_phase0(step_layer(0));
        if (x_by_copy(0)) issue_x(0);
    }
    uint32_t ph = 0;  // parity of the phase each mbarrier is in

    for (int s = 0; s < p.n_steps; ++s) {
        uint64_t* trace = (p.trace && s == p.n_steps / 2) ? p.trace + (size_t)c * kTraceSlots : nullptr;
#define TRACE(i) do { if (trace && tid == 0) trace[i] = global_ns(); } while (0)
        TRACE(0);
        const moe_b200_layer* Ls = step_layer(s);
        const uint32_t gen = (uint32_t)G * (uint32_t)(s + 1);  // counter value once step s is done
        const uint32_t tag = seq0 + (uint32_t)s + 1u;             // exchange-word tag of step s
        int sflags = 0;
        const float* xin = p.x;
        float* yout = p.y;
        int32_t* ids_out = p.ids_out;
        float* w_out = p.w_out;
        if (p.steps) {
            const moe_b200_step& st = p.steps[s];
            sflags = st.flags;
            xin = (sflags & MOE_B200_STEP_CHAIN) && s > 0 ? p.steps[s - 1].y : st.x;
            yout = st.y;
            ids_out = st.topk_ids;
            w_out = st.topk_weights;
        }
        const int buf = s & 1;
        uint64_t* scores = p.scores + (size_t)buf * E;
        uint64_t* act_r = p.act_r + (size_t)buf * K * I;
        uint64_t* act_s = p.act_s + (size_t)buf * Imax;
        uint64_t* sgp = p.sg + buf;
        const bool chain = (sflags & MOE_B200_STEP_CHAIN) && s > 0;
        const bool block = (sflags & MOE_B200_STEP_BLOCK) != 0;

        // ---- the token (after the previous step, whose output it is, when chained)
        if (chain) {
            if (tid == 0 && !wait_flag(p.ctr + C_DONE, (uint32_t)G * (uint32_t)s, kWaitPolls))
                set_error(p.ctr, ST_TIMEOUT);
            __syncthreads();
            for (int i = tid; i < H; i += kFusedThreads) x32[i] = __ldcg(xin + i);
        } else if (x_by_copy(s)) {
            if (tid == 0 && !mbar_wait(&bars[kXBar], (ph >> kXBar) & 1u, kWaitPolls))
                set_error(p.ctr, ST_TIMEOUT);
            ph ^= 1u << kXBar;
        } else {
            for (int i = tid; i < H; i += kFusedThreads) x32[i] = xin[i];
        }
        __syncthreads();
        if (block) {
            // h = x + rmsnorm16(x); the MoE input is rmsnorm16(h)
            // (reference TransformerBlock.forward with an identity mixer,
            // src/flash_moe/transformer.py:229-247; RMSNorm norm.py:28-30)
            float ss = 0.f;
            for (int i = tid; i < H; i += kFusedThreads) ss = fmaf(x32[i], x32[i], ss);
            ss = block_sum(ss, s_part);
            const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps));
            float ss2 = 0.f;
            for (int i = tid; i < H; i += kFusedThreads) {
                const float hv = __fadd_rn(x32[i], round16(__fdiv_rn(x32[i], rms)));
                h32[i] = hv;
                ss2 = fmaf(hv, hv, ss2);
            }
            ss2 = block_sum(ss2, s_part);
            const float rms2 = sqrtf(__fadd_rn(__fdiv_rn(ss2, (float)H), p.eps));
            for (int i = tid; i < H; i += kFusedThreads) x32[i] = round16(__fdiv_rn(h32[i], rms2));
            __syncthreads();
        }
        TRACE(1);

        // ---- router scores (rows [r0, r1)): each row split over nw/R warps,
        // partial sums combined in a fixed order (deterministic)
        if (tid == 0 && !mbar_wait(&bars[0], ph & 1u, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        ph ^= 1u;
        __syncthreads();
        TRACE(2);
        {
            const float* router_s = reinterpret_cast<const float*>(sm + p.o_router);
            const float* bias = Ls->router_bias;
            const int R = r1 - r0;
            if (R > 0 && R <= nw) {
                const int spr = nw / R;
                const int row = warp / spr, sl = warp % spr;
                if (row < R) {
                    const int cw = (H / spr) & ~3;  // 16-byte aligned slices
                    const int cc0 = sl * cw, cn = (sl == spr - 1) ? H - cc0 : cw;
                    float acc = dot_f32_warp(router_s + (size_t)row * H + cc0, x32 + cc0, cn, lane);
                    if (lane == 0) s_part[warp] = acc;
                }
                __syncthreads();
                if (tid < R) {
                    float acc = 0.f;
                    for (int q = 0; q < spr; ++q) acc += s_part[tid * spr + q];
                    if (bias) acc = __fadd_rn(acc, bias[r0 + tid]);
                    st_word_gpu(scores + r0 + tid, acc, tag);
                }
            } else {
                for (int rr = warp; rr < R; rr += nw) {
                    float acc = dot_f32_warp(router_s + (size_t)rr * H, x32, H, lane);
                    if (lane == 0) {
                        if (bias) acc = __fadd_rn(acc, bias[r0 + rr]);
                        st_word_gpu(scores + r0 + rr, acc, tag);
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0 && !tagged) red_release_add(p.ctr + C_ROUTER, 1);
        TRACE(3);

        // ---- the token quantised for the integer dot products; shared gate
        for (int b = warp; b < H / 256; b += nw) quantize_block_warp(x32, xq, b);
        TRACE(23);
        if (Is && c == 0 && warp == nw - 1) {
            const float* ginp = Ls->shared_gate_inp;
            float acc = 0.f;
            for (int i = lane; i < H; i += 32) acc = fmaf(x32[i], ginp[i], acc);
            acc = warp_sum(acc);
            if (lane == 0) st_word_gpu(sgp, shared_sigmoid(acc), tag);
        }
        __syncthreads();
        TRACE(24);
        XLane xl;
        load_xlane(xl, xq, pr_h >> 2, pr_h & 3);
        TRACE(25);

        // ---- routing (every CTA, identically): the selection first, so the
        // routed copies start at once; the weights later, off that path
        if (!tagged) {
            if (tid == 0 && !wait_flag(p.ctr + C_ROUTER, gen, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
            __syncthreads();
        }
        TRACE(5);
        if (E > 256) {
            bool ok = true;
            for (int e = tid; e < E; e += kFusedThreads) s_scores[e] = wait_word_gpu(scores + e, tag, kWaitPolls, ok);
            if (!ok) set_error(p.ctr, ST_TIMEOUT);
            __syncthreads();
        }
        uint32_t sel_k = 0;
        int sel_id = 0;
        if (warp == 0) {
            if (E <= 256) {
                uint32_t kk[8];
                int kid[8];
                if (!load_score_words(scores, E, tag, kWaitPolls,
                                      reinterpret_cast<uint32_t*>(s_scores), kk, kid) &&
                    lane == 0)
                    set_error(p.ctr, ST_TIMEOUT);
                topk_select_warp(kk, kid, K, sel_k, sel_id, trace);
                if (lane < K) s_ids[lane] = sel_id;
            } else {
                topk_softmax_warp(s_scores, s_taken, E, K, s_ids, s_w);
            }
            __syncwarp();
            // the selections this GPU holds, in top-k order
            const int e = lane < K ? s_ids[lane] : -1;
            const bool held = lane < K && e >= ebeg && e < ebeg + ecnt;
            const uint32_t hb = __ballot_sync(0xffffffffu, held);
            if (held) s_act[__popc(hb & ((1u << lane) - 1u))] = lane;
            if (lane == 0) *s_nact = __popc(hb);
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
        const int nchunks = (nrows + CR - 1) / CR;
        // issued by the lanes of warp 0 in parallel: lane q < nchunks chunk q;
        // the down rows (lane 16 + a: slot a) once the last gate/up chunk has
        // landed, so they do not compete with the gate/up bytes, which are
        // needed first
        auto issue_down = [&]() {
            if (lane == 16) mbar_arrive_expect_tx(&bars[2], (uint32_t)(A * nh * rb_down));
            if (lane >= 16 && lane - 16 < A && nh > 0) {
                const int a = lane - 16;
                const int64_t e = s_ids[s_act[a]] - ebeg;
                bulk_g2s(sm + p.o_rdown + (int64_t)a * p.max_out_rows * rb_down,
                         Ls->down + e * st_down + h0 * rb_down, (uint32_t)(nh * rb_down), &bars[2]);
            }
        };
        if (warp == 0) {
            const uint8_t* gate = Ls->gate;
            const uint8_t* up = Ls->up;
            if (lane < nchunks) {
                const int q = lane, q0 = q * CR, q1 = min(nrows, q0 + CR);
                mbar_arrive_expect_tx(&bars[3 + q], (uint32_t)((q1 - q0) * (rb_gate + rb_up)));
                for (int f = f0 + q0; f < f0 + q1;) {
                    const int a = f / I, r = f % I;
                    const int n = min(f0 + q1 - f, I - r);
                    const int64_t e = s_ids[s_act[a]] - ebeg;
                    bulk_g2s(sm + p.o_rgate + (int64_t)(f - f0) * rb_gate, gate + e * st_gate + r * rb_gate,
                             (uint32_t)(n * rb_gate), &bars[3 + q]);
                    bulk_g2s(sm + p.o_rup + (int64_t)(f - f0) * rb_up, up + e * st_up + r * rb_up,
                             (uint32_t)(n * rb_up), &bars[3 + q]);
                    f += n;
                }
            }
            // routing weights (float64 softmax over the selections), needed
            // only by the combine
            if (E <= 256) topk_weights_warp(sel_k, sel_id, K, s_ids, s_w);
            if (c == 0 && lane < K) {
                if (ids_out) ids_out[lane] = s_ids[lane];
                if (w_out) w_out[lane] = s_w[lane];
            }
            TRACE(15);
        }

        // ---- shared expert gate/up (x is the token), while the routed rows
        // are in flight; rows go to the last warps first (warp 0 issues the
        // copies).  Its counter is released with the gate/up one.
        if (Is) {
            if (!mbar_wait(&bars[1], (ph >> 1) & 1u, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
            ph ^= 2u;
            const int rpw = 32 / lpr_h;
            for (int rb = (nw - 1 - warp) * rpw; rb < s1 - s0; rb += nw * rpw) {
                const int rr = rb + sub_h;
                const bool ok = rr < s1 - s0;
                const int rs = ok ? rr : 0;
                float g = qdot_t<SGU>(L0.shared_gate_type, sm + p.o_sgate + rs * rb_sg, pr_h >> 2, pr_h & 3, xl);
                float u = qdot_t<SGU>(L0.shared_up_type, sm + p.o_sup + rs * rb_su, pr_h >> 2, pr_h & 3, xl);
                g = group_sum(g, lpr_h);
                u = group_sum(u, lpr_h);
                if (ok && pr_h == 0) st_word_gpu(act_s + s0 + rr, (g * shared_sigmoid(g)) * u, tag);
            }
        }
        TRACE(4);

        // ---- routed gate/up, chunk by chunk
        {
            const int rpw = 32 / lpr_h;
            int waited = -1;
            for (int rb = warp * rpw; rb < nrows; rb += nw * rpw) {
                const int qlast = min(rb + rpw - 1, nrows - 1) / CR;
                while (waited < qlast) {
                    ++waited;
                    if (!mbar_wait(&bars[3 + waited], (ph >> (3 + waited)) & 1u, kWaitPolls) && lane == 0)
                        set_error(p.ctr, ST_TIMEOUT);
                    if (waited < 2) TRACE(16 + waited);
                    if (warp == 0 && waited == nchunks - 1) issue_down();
                }
                const int rr = rb + sub_h;
                const bool ok = rr < nrows;
                const int rs = ok ? rr : 0;
                float g = qdot_t<GU>(L0.gate_type, sm + p.o_rgate + rs * rb_gate, pr_h >> 2, pr_h & 3, xl);
                float u = qdot_t<GU>(L0.up_type, sm + p.o_rup + rs * rb_up, pr_h >> 2, pr_h & 3, xl);
                g = group_sum(g, lpr_h);
                u = group_sum(u, lpr_h);
                if (ok && pr_h == 0) {
                    const float sgm = 1.0f / (1.0f + expf(-g));
                    st_word_gpu(act_r + f0 + rr, (g * sgm) * u, tag);
                }
                if (rb == 0) TRACE(18);
            }
            // every chunk barrier must have completed before the CTA moves on
            // (its copies write shared memory)
            for (int q = waited + 1; q < nchunks; ++q) {
                if (!mbar_wait(&bars[3 + q], (ph >> (3 + q)) & 1u, kWaitPolls) && lane == 0)
                    set_error(p.ctr, ST_TIMEOUT);
                if (warp == 0 && q == nchunks - 1) issue_down();
            }
            if (warp == 0 && nchunks == 0) issue_down();
            ph ^= ((1u << nchunks) - 1u) << 3;
        }
        TRACE(7);
        __syncthreads();
        TRACE(8);
        if (tid == 0 && !tagged) {
            if (Is) red_release_add(p.ctr + C_SHARED, 1);
            red_release_add(p.ctr + C_GATEUP, 1);
            if (Is && !wait_flag(p.ctr + C_SHARED, gen, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
            if (!wait_flag(p.ctr + C_GATEUP, gen, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        }
        __syncthreads();
        TRACE(9);

        // ---- activations, vector by vector: warp w gathers vector v = w
        // (+16, ...) -- routed slot v < A (I values) or the shared vector
        // v == A (Is values and the shared gate) -- from the exchange words,
        // quantises it and marks it ready (s_ready[v] = tag).  A down item
        // starts as soon as its vector is ready, so the exchange of the late
        // vectors overlaps the down rows of the early ones; the shared
        // vector, whose rows were done first, leads.
        float* act32 = reinterpret_cast<float*>(sm + p.o_act);
        const uint32_t qb = qvec_bytes(Imax);
        const int nvec = A + (Is ? 1 : 0);
        for (int v = warp; v < nvec; v += nw) {
            const int n = v < A ? I : Is;
            const uint64_t* src = v < A ? act_r + (size_t)v * I : act_s;
            float* dst = act32 + v * Imax;
            bool ok = true;
            for (int j0 = 2 * lane; j0 < n; j0 += 2 * 32 * kGatherPairs) {
                uint32_t pend = 0;
#pragma unroll
                for (int q = 0; q < kGatherPairs; ++q)
                    if (j0 + 64 * q < n) pend |= 1u << q;
                for (uint32_t round = 0; pend != 0u; ++round) {
                    if (round == kWaitPolls) {
                        ok = false;
                        break;
                    }
                    ulonglong2 wv[kGatherPairs];
#pragma unroll
                    for (int q = 0; q < kGatherPairs; ++q)
                        wv[q] = ((pend >> q) & 1u) ? ld_word2_gpu(src + j0 + 64 * q) : make_ulonglong2(0ull, 0ull);
#pragma unroll
                    for (int q = 0; q < kGatherPairs; ++q) {
                        if (((pend >> q) & 1u) && (uint32_t)(wv[q].x >> 32) == tag &&
                            (uint32_t)(wv[q].y >> 32) == tag) {
                            pend &= ~(1u << q);
                            *reinterpret_cast<float2*>(dst + j0 + 64 * q) =
                                make_float2(__uint_as_float((uint32_t)wv[q].x), __uint_as_float((uint32_t)wv[q].y));
                        }
                    }
                }
                if (!ok) break;
            }
            if (v == A && lane == 0) *s_sg = wait_word_gpu(sgp, tag, kWaitPolls, ok);
            if (!__all_sync(0xffffffffu, ok) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
            __syncwarp();
            if (v == 0) TRACE(19);
            for (int b = 0; b < n / 256; ++b) quantize_block_warp(dst, qvec_at(sm + p.o_aq + v * qb, n), b);
            __syncwarp();
            __threadfence_block();
            if (lane == 0) s_ready[v] = tag;
            if (v == 0) TRACE(20);
        }
        // the down rows of this CTA (every warp checks the copy)
        if (!mbar_wait(&bars[2], (ph >> 2) & 1u, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
        ph ^= 4u;
        TRACE(10);

        // ---- down rows [h0, h1) of every vector: item = (routed vector, pair
        // of row groups), the activation codes loaded once per item; the
        // shared vector's row groups come first, one per item
        {
            const int rpw_i = 32 / p.lpr_i, rpw_s = 32 / p.lpr_is;
            const int ng_i = (nh + rpw_i - 1) / rpw_i, ng_s = Is ? (nh + rpw_s - 1) / rpw_s : 0;
            const int np_i = (ng_i + 1) / 2, np_s = ng_s;
            for (int it = warp; it < A * np_i + np_s; it += nw) {
                const bool sh = it < np_s;
                const int v = sh ? A : (it - np_s) / np_i;
                const int gp = sh ? it : (it - np_s) % np_i;
                const int lpr = sh ? p.lpr_is : p.lpr_i;
                const int ng = sh ? ng_s : ng_i;
                const int rpw = 32 / lpr, sub = lane / lpr, pr = lane % lpr;
                const int type = sh ? L0.shared_down_type : L0.down_type;
                const int64_t rb = sh ? rb_sd : rb_down;
                const uint8_t* rows = sh ? sm + p.o_sdown : sm + p.o_rdown + (int64_t)v * p.max_out_rows * rb_down;
                const int n = sh ? Is : I;
                {
                    uint32_t i = 0;
                    while (s_ready[v] != tag && ++i < kWaitPolls) {
                    }
                    if (i == kWaitPolls && lane == 0) set_error(p.ctr, ST_TIMEOUT);
                    __syncwarp();
                    __threadfence_block();
                }
                XLane xa;
                load_xlane(xa, qvec_at(sm + p.o_aq + v * qb, n), pr >> 2, pr & 3);
#pragma unroll
                for (int gg = 0; gg < 2; ++gg) {
                    const int gi = sh ? (gg == 0 ? gp : ng) : 2 * gp + gg;
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
        // ---- weighted sum in top-k order, + shared (moe_layer.py:85-86, 102-105);
        // block steps add the residual h to the binary16-rounded MoE output
        // (transformer.py:192-204, 229-247)
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
            if (block) comb = __fadd_rn(h32[h0 + rr], round16(comb));
            yout[h0 + rr] = comb;
        }
        __syncthreads();
        TRACE(12);
#undef TRACE
        if (tid == 0) {
            red_release_add(p.ctr + C_DONE, 1);
            // the router and shared-expert regions are free: the next step's
            // rows load while this CTA waits for the others
            if (s + 1 < p.n_steps) {
                issue_phase0(step_layer(s + 1));
                if (x_by_copy(s + 1)) issue_x(s + 1);
            }
        }
    }
    // ---- exit: the last CTA resets the counters for the next launch
    if (tid == 0) {
        __threadfence();
        const uint32_t t = atomicAdd(p.ctr + C_EXIT, 1u);
        if (t == (uint32_t)G - 1) {
            p.ctr[C_ROUTER] = 0;
            p.ctr[C_SHARED] = 0;
            p.ctr[C_GATEUP] = 0;
            p.ctr[C_DONE] = 0;
            p.ctr[C_EXIT] = 0;
            p.ctr[C_SEQ] = seq0 + (uint32_t)p.n_steps;
            if (p.err_out) {
                *p.err_out = atomicExch(reinterpret_cast<int*>(p.ctr + C_ERROR), 0);
                __threadfence_system();
            }
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
    // counters, then two buffers (step parity) of scores, routed and shared
    // activations and the shared gate
    return 256 + align_up((size_t)2 * L->n_experts * 8) +
           align_up((size_t)2 * L->top_k * L->intermediate * 8) + align_up((size_t)2 * Imax * 8) + 256;
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
    p.o_h32 = take((uint64_t)H * 4);
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
    p.o_misc = take(512 + ((5 * E + 15) & ~15) + (uint64_t)(K + 1) * p.max_out_rows * 4 +
                    4 * (kMaxTopK + 1));
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

using FusedFn = void (*)(FusedParams);

// Parameters and kernel instance of one launch of the fused kernel: a
// single step (steps null: the token x through layer *L) or n_steps steps
// from the device tables.  False when the layer does not fit the plan.
static cudaError_t fused_prepare(const moe_b200_layer* L, int flags, const float* x, float* y,
                                 int32_t* ids_out, float* w_out, const moe_b200_layer* layers,
                                 const moe_b200_step* steps, int n_steps, float eps, void* ws,
                                 FusedParams& p, FusedFn& fn, bool* ok) {
    *ok = false;
    const bool shared = L->shared_intermediate > 0 && !(flags & MOE_B200_NO_SHARED);
    memset(&p, 0, sizeof(p));
    p.L = *L;
    const int G = sm_count();
    if (!fused_plan(L, shared, G, p)) return cudaSuccess;
    struct Instance {
        int gu, dn, sgu, sdn;
        FusedFn fn;
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
    fn = kInstances[pick].fn;
    char* base = static_cast<char*>(ws);
    p.x = x;
    p.y = y;
    p.ids_out = ids_out;
    p.w_out = w_out;
    p.layers = layers;
    p.steps = steps;
    p.n_steps = steps ? n_steps : 1;
    p.eps = eps;
    p.ctr = reinterpret_cast<uint32_t*>(base);
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate : L->intermediate;
    size_t off = 256;
    p.scores = reinterpret_cast<uint64_t*>(base + off);
    off += align_up((size_t)2 * L->n_experts * 8);
    p.act_r = reinterpret_cast<uint64_t*>(base + off);
    off += align_up((size_t)2 * L->top_k * L->intermediate * 8);
    p.act_s = reinterpret_cast<uint64_t*>(base + off);
    off += align_up((size_t)2 * Imax * 8);
    p.sg = reinterpret_cast<uint64_t*>(base + off);
    p.trace = (tl_trace && tl_trace_cap >= G) ? tl_trace : nullptr;
    *ok = true;
    return cudaSuccess;
}

static cudaError_t fused_launch(const moe_b200_layer* L, int flags, const float* x, float* y,
                                int32_t* ids_out, float* w_out, const moe_b200_layer* layers,
                                const moe_b200_step* steps, int n_steps, float eps, void* ws,
                                cudaStream_t stream, bool* launched) {
    *launched = false;
    FusedParams p;
    FusedFn fn = nullptr;
    bool ok = false;
    cudaError_t e = fused_prepare(L, flags, x, y, ids_out, w_out, layers, steps, n_steps, eps, ws,
                                  p, fn, &ok);
    if (e != cudaSuccess || !ok) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.G);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = p.total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, fn, p);
    if (e == cudaSuccess) *launched = true;
    return e;
}

// x rows from host memory the device can read (pinned, mapped) into device
// staging rows: one 16-byte word per thread.
__global__ void __launch_bounds__(256) k_copy_in(const float4* __restrict__ src,
                                                 float4* __restrict__ dst, int n4) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n4) dst[i] = src[i];
}

// Per-thread graphs of (copy-in kernel -> fused kernel) for synchronous
// single-token calls with host buffers: a graph launch reaches the GPU
// sooner than a direct cooperative launch.  The caller's buffers are the
// library's fixed pinned staging rows, so a graph's parameters depend only on
// the layer, the workspace and the device: one graph per such combination is
// kept (at most kHostGraphs per thread, oldest dropped first) and replayed
// without parameter updates.  A thread's graphs are left to the driver's
// clean-up at process exit.
constexpr size_t kHostGraphs = 64;

struct HostGraphKey {
    int dev;
    FusedFn fn;
    FusedParams p;
    const float4* src;
    float4* dst;
    int n4;
};

struct HostGraph {
    HostGraphKey key;
    cudaGraph_t g;
    cudaGraphExec_t ge;
};

cudaError_t launch_decode_fused_host(const moe_b200_layer* L, int flags, const float* x_host,
                                     float* x_stage, float* y_host, int32_t* ids_host,
                                     float* w_host, int* err_host, void* ws, cudaStream_t stream,
                                     bool* launched) {
    *launched = false;
    HostGraphKey k;
    memset(&k, 0, sizeof(k));
    bool ok = false;
    cudaError_t e = fused_prepare(L, flags, x_stage, y_host, ids_host, w_host, nullptr, nullptr, 1,
                                  0.f, ws, k.p, k.fn, &ok);
    if (e != cudaSuccess || !ok) return e;
    k.p.err_out = err_host;
    if ((e = cudaGetDevice(&k.dev)) != cudaSuccess) return e;
    k.n4 = L->hidden / 4;
    k.src = reinterpret_cast<const float4*>(x_host);
    k.dst = reinterpret_cast<float4*>(x_stage);
    static thread_local std::vector<HostGraph> cache;
    for (size_t i = 0; i < cache.size(); ++i) {
        if (memcmp(&cache[i].key, &k, sizeof(k)) == 0) {
            e = cudaGraphLaunch(cache[i].ge, stream);
            if (e == cudaSuccess) *launched = true;
            return e;
        }
    }
    HostGraph hg;
    hg.key = k;
    hg.g = nullptr;
    hg.ge = nullptr;
    void* cargs[] = {&hg.key.src, &hg.key.dst, &hg.key.n4};
    cudaKernelNodeParams cp = {};
    cp.func = reinterpret_cast<void*>(k_copy_in);
    cp.gridDim = dim3((k.n4 + 255) / 256);
    cp.blockDim = dim3(256);
    cp.kernelParams = cargs;
    void* fargs[] = {&hg.key.p};
    cudaKernelNodeParams fp = {};
    fp.func = reinterpret_cast<void*>(k.fn);
    fp.gridDim = dim3(k.p.G);
    fp.blockDim = dim3(kFusedThreads);
    fp.sharedMemBytes = k.p.total;
    fp.kernelParams = fargs;
    cudaGraphNode_t copy = nullptr, fused = nullptr;
    e = cudaGraphCreate(&hg.g, 0);
    if (e == cudaSuccess) e = cudaGraphAddKernelNode(&copy, hg.g, nullptr, 0, &cp);
    if (e == cudaSuccess) e = cudaGraphAddKernelNode(&fused, hg.g, &copy, 1, &fp);
    if (e == cudaSuccess) {
        cudaLaunchAttributeValue v = {};
        v.cooperative = 1;
        e = cudaGraphKernelNodeSetAttribute(fused, cudaLaunchAttributeCooperative, &v);
    }
    if (e == cudaSuccess) e = cudaGraphInstantiate(&hg.ge, hg.g, 0);
    if (e != cudaSuccess) {
        if (hg.ge) cudaGraphExecDestroy(hg.ge);
        if (hg.g) cudaGraphDestroy(hg.g);
        return e;
    }
    if (cache.size() >= kHostGraphs) {
        cudaGraphExecDestroy(cache.front().ge);
        cudaGraphDestroy(cache.front().g);
        cache.erase(cache.begin());
    }
    cache.push_back(hg);
    e = cudaGraphLaunch(hg.ge, stream);
    if (e == cudaSuccess) *launched = true;
    return e;
}

cudaError_t launch_decode_fused(const moe_b200_layer* L, int flags, const float* x, float* y,
                                int32_t* ids_out, float* w_out, void* ws, cudaStream_t stream,
                                bool* launched) {
    return fused_launch(L, flags, x, y, ids_out, w_out, nullptr, nullptr, 1, 0.f, ws, stream,
                        launched);
}

cudaError_t launch_decode_steps(const moe_b200_layer* L0, const moe_b200_layer* layers,
                                const moe_b200_step* steps, int n_steps, float eps, void* ws,
                                cudaStream_t stream, bool* launched) {
    return fused_launch(L0, L0->flags, nullptr, nullptr, nullptr, nullptr, layers, steps, n_steps,
                        eps, ws, stream, launched);
}

}  // namespace moeb200
