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

constexpr int kMaxChunks = 8;             // routed gate/up copy chunks (mbarriers 3..10)
constexpr int kXBar = 3 + kMaxChunks;      // mbarrier of the prefetched token
constexpr int kSdBar = kXBar + 1;          // mbarrier of the shared-expert down rows
constexpr int kNumBars = kSdBar + 1;
constexpr int kGatherWords = 10;           // exchange words a thread has in flight per poll round

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
    uint64_t* scores;        // [2][S]       exchange words (buffer = step parity)
    uint64_t* act_r;         // [2][K x I]
    uint64_t* act_s;         // [2][Imax]
    uint64_t* yw;            // [2][H]       the layer output of a step a CHAIN step reads
    uint64_t* trace;         // [G x 32] phase timestamps of step n_steps / 2 (ns), or null
    int* err_out;            // null, or a host-visible word that receives (and clears) the
                             // error word at exit
    int G;
    int S;                   // score slots: max(E, G), so every CTA writes one each step
    int with_shared;
    int max_router_rows, max_sgu_rows, max_out_rows, max_rgu_rows;
    int lpr_h, lpr_i, lpr_is;
    int chunk_rows;
    uint32_t o_x32, o_h32, o_xq, o_router, o_ginp, o_sgate, o_sup, o_sdown, o_rgate, o_rup, o_rdown;
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
    const int H = L0.hidden, I = L0.intermediate, E = L0.n_experts, K = L0.top_k, S = p.S;
    const int Is = p.with_shared ? L0.shared_intermediate : 0;
    const int ebeg = L0.expert_begin, ecnt = L0.expert_count;
    const int64_t rb_gate = row_bytes(L0.gate_type, H), rb_up = row_bytes(L0.up_type, H);
    const int64_t rb_down = row_bytes(L0.down_type, I);
    const int64_t st_gate = rb_gate * I, st_up = rb_up * I, st_down = rb_down * H;
    const int64_t rb_sg = Is ? row_bytes(L0.shared_gate_type, H) : 0;
    const int64_t rb_su = Is ? row_bytes(L0.shared_up_type, H) : 0;
    const int64_t rb_sd = Is ? row_bytes(L0.shared_down_type, Is) : 0;
    const int Imax = max(I, Is);
    const uint32_t seq0 = ld_acquire(p.ctr + C_SEQ);

    uint64_t* bars = reinterpret_cast<uint64_t*>(sm + p.o_misc);       // [kNumBars]
    int* s_ids = reinterpret_cast<int*>(sm + p.o_misc + 128);          // [16]
    float* s_w = reinterpret_cast<float*>(sm + p.o_misc + 192);        // [16]
    int* s_act = reinterpret_cast<int*>(sm + p.o_misc + 256);          // [16] active slots
    int* s_nact = reinterpret_cast<int*>(sm + p.o_misc + 320);
    float* s_sg = reinterpret_cast<float*>(sm + p.o_misc + 324);
    float* s_part = reinterpret_cast<float*>(sm + p.o_misc + 384);     // [32] partial sums
    float* s_scores = reinterpret_cast<float*>(sm + p.o_misc + 512);   // [S]
    float* s_vout = reinterpret_cast<float*>(sm + p.o_misc + 512 + ((5 * S + 15) & ~15));
    float* x32 = reinterpret_cast<float*>(sm + p.o_x32);
    float* h32 = reinterpret_cast<float*>(sm + p.o_h32);

    const int r0 = part(S, c, G), r1 = part(S, c + 1, G);  // score slots; rows < E are router rows
    const int re1 = min(r1, E), nr = max(0, re1 - r0);      // router rows of this CTA
    const int s0 = part(Is, c, G), s1 = part(Is, c + 1, G);
    const int h0 = part(H, c, G), h1 = part(H, c + 1, G);
    const int nh = h1 - h0;
    const int lpr_h = p.lpr_h, sub_h = lane / lpr_h, pr_h = lane % lpr_h;

    auto step_layer = [&](int s) -> const moe_b200_layer* {
        return p.steps ? p.layers + p.steps[s].layer : &p.L;
    };
    // The resident rows of a step, each set on its own mbarrier, so that each
    // is reissued for the next step as soon as this step is done with it:
    // router rows + shared gate vector (bars[0]), shared gate/up rows
    // (bars[1]), shared down rows (bars[kSdBar]).
    auto issue_router = [&](const moe_b200_layer* Ls) {
        const uint32_t rbytes = (uint32_t)(nr * H * 4);
        // the gate vector by TMA when 16-byte aligned, else read in place
        const uint32_t gbytes = (Is && Ls->shared_gate_inp && (((uintptr_t)Ls->shared_gate_inp) & 15u) == 0)
                                    ? (uint32_t)(H * 4) : 0u;
        mbar_arrive_expect_tx(&bars[0], rbytes + gbytes);
        if (nr > 0) bulk_g2s(sm + p.o_router, Ls->router + (size_t)r0 * H, rbytes, &bars[0]);
        if (gbytes) bulk_g2s(sm + p.o_ginp, Ls->shared_gate_inp, gbytes, &bars[0]);
    };
    auto issue_sgu = [&](const moe_b200_layer* Ls) {
        mbar_arrive_expect_tx(&bars[1], (uint32_t)((s1 - s0) * (rb_sg + rb_su)));
        if (s1 > s0) {
            bulk_g2s(sm + p.o_sgate, Ls->shared_gate + s0 * rb_sg, (uint32_t)((s1 - s0) * rb_sg), &bars[1]);
            bulk_g2s(sm + p.o_sup, Ls->shared_up + s0 * rb_su, (uint32_t)((s1 - s0) * rb_su), &bars[1]);
        }
    };
    auto issue_sdown = [&](const moe_b200_layer* Ls) {
        mbar_arrive_expect_tx(&bars[kSdBar], (uint32_t)(nh * rb_sd));
        if (nh > 0) bulk_g2s(sm + p.o_sdown, Ls->shared_down + h0 * rb_sd, (uint32_t)(nh * rb_sd), &bars[kSdBar]);
    };

    // A step's token comes by TMA (issued before the step begins) unless it
    // is the previous step's output or not 16-byte aligned.
    auto chained = [&](int s) -> bool {
        return p.steps && s > 0 && (p.steps[s].flags & MOE_B200_STEP_CHAIN);
    };
    auto step_x = [&](int s) -> const float* { return p.steps ? p.steps[s].x : p.x; };
    auto x_by_copy = [&](int s) -> bool { return !chained(s) && (((uintptr_t)step_x(s)) & 15u) == 0; };
    auto issue_x = [&](int s) {
        mbar_arrive_expect_tx(&bars[kXBar], (uint32_t)(H * 4));
        bulk_g2s(x32, step_x(s), (uint32_t)(H * 4), &bars[kXBar]);
    };
    // bounded wait of every thread on an mbarrier phase (one poller, then the CTA)
    uint32_t ph = 0;  // parity of the phase each mbarrier is in
    auto cta_wait = [&](int b) {
        if (tid == 0 && !mbar_wait(&bars[b], (ph >> b) & 1u, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        ph ^= 1u << b;
        __syncthreads();
    };

    if (tid == 0) {
        for (int i = 0; i < kNumBars; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        const moe_b200_layer* L1 = step_layer(0);
        issue_router(L1);
        if (Is) {
            issue_sgu(L1);
            issue_sdown(L1);
        }
        if (x_by_copy(0)) issue_x(0);
    }

    for (int s = 0; s < p.n_steps; ++s) {
        uint64_t* trace = (p.trace && s == p.n_steps / 2) ? p.trace + (size_t)c * kTraceSlots : nullptr;
#define TRACE(i) do { if (trace && tid == 0) trace[i] = global_ns(); } while (0)
        TRACE(0);
        const moe_b200_layer* Ls = step_layer(s);
        const uint32_t tag = seq0 + (uint32_t)s + 1u;  // exchange-word tag of step s
        int sflags = 0;
        const float* xin = p.x;
        float* yout = p.y;
        int32_t* ids_out = p.ids_out;
        float* w_out = p.w_out;
        if (p.steps) {
            const moe_b200_step& st = p.steps[s];
            sflags = st.flags;
            xin = st.x;
            yout = st.y;
            ids_out = st.topk_ids;
            w_out = st.topk_weights;
        }
        const int buf = s & 1;
        uint64_t* scores = p.scores + (size_t)buf * S;
        uint64_t* act_r = p.act_r + (size_t)buf * K * I;
        uint64_t* act_s = p.act_s + (size_t)buf * Imax;
        const bool chain = chained(s);
        const bool block = (sflags & MOE_B200_STEP_BLOCK) != 0;
        const bool next_chains = s + 1 < p.n_steps && chained(s + 1);
        const moe_b200_layer* Ln = s + 1 < p.n_steps ? step_layer(s + 1) : nullptr;

        // ---- the token: the previous step's output words (CHAIN), the
        // prefetched copy, or direct loads
        if (chain) {
            const uint64_t* src = p.yw + (size_t)(buf ^ 1) * H;
            bool ok = true;
            for (int j0 = tid; j0 < H; j0 += kFusedThreads * kGatherWords) {
                uint32_t pend = 0;
#pragma unroll
                for (int q = 0; q < kGatherWords; ++q)
                    if (j0 + kFusedThreads * q < H) pend |= 1u << q;
                for (uint32_t round = 0; pend != 0u; ++round) {
                    if (round == kWaitPolls) {
                        ok = false;
                        break;
                    }
                    uint64_t wv[kGatherWords];
#pragma unroll
                    for (int q = 0; q < kGatherWords; ++q)
                        wv[q] = ((pend >> q) & 1u) ? ld_word_gpu(src + j0 + kFusedThreads * q) : 0ull;
#pragma unroll
                    for (int q = 0; q < kGatherWords; ++q)
                        if (((pend >> q) & 1u) && (uint32_t)(wv[q] >> 32) == tag - 1u) {
                            pend &= ~(1u << q);
                            x32[j0 + kFusedThreads * q] = __uint_as_float((uint32_t)wv[q]);
                        }
                }
            }
            if (!ok) set_error(p.ctr, ST_TIMEOUT);
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
#pragma unroll 1
            for (int i = tid; i < H; i += kFusedThreads) ss = fmaf(x32[i], x32[i], ss);
            ss = block_sum(ss, s_part);
            const float rms = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)H), p.eps));
            float ss2 = 0.f;
#pragma unroll 1
            for (int i = tid; i < H; i += kFusedThreads) {
                const float hv = __fadd_rn(x32[i], round16(__fdiv_rn(x32[i], rms)));
                h32[i] = hv;
                ss2 = fmaf(hv, hv, ss2);
            }
            ss2 = block_sum(ss2, s_part);
            const float rms2 = sqrtf(__fadd_rn(__fdiv_rn(ss2, (float)H), p.eps));
#pragma unroll 1
            for (int i = tid; i < H; i += kFusedThreads) x32[i] = round16(__fdiv_rn(h32[i], rms2));
            __syncthreads();
        }
        TRACE(1);

        // ---- router rows [r0, re1) and the shared gate x . w_inp (every CTA
        // computes the gate itself: one more row of the same dot), each row
        // split over nw / R warps, partial sums combined in a fixed order
        // (deterministic); score slots [re1, r1) carry no score
        cta_wait(0);
        TRACE(2);
        {
            const float* router_s = reinterpret_cast<const float*>(sm + p.o_router);
            const bool ginp_tma = ((((uintptr_t)Ls->shared_gate_inp) & 15u) == 0);
            const float* ginp_s = ginp_tma ? reinterpret_cast<const float*>(sm + p.o_ginp) : Ls->shared_gate_inp;
            const float* bias = Ls->router_bias;
            const bool with_gate = Is && Ls->shared_gate_inp;
            // warps 0..nw-2: the router rows (<= nw - 1 of them, fused_plan);
            // warp nw-1: the gate, lane-strided like the multi-token kernel
            // (same summation order, so the two kernels' gates agree bit for bit)
            const int nwr = nw - 1;
            if (nr > 0) {
                const int spr = nwr / nr;
                const int row = warp / spr, sl = warp % spr;
                if (warp < nwr && row < nr) {
                    const int cw = (H / spr) & ~3;  // 16-byte aligned slices
                    const int cc0 = sl * cw, cn = (sl == spr - 1) ? H - cc0 : cw;
                    const float* rp = router_s + (size_t)row * H + cc0;
                    const float* xp = x32 + cc0;
                    float acc = 0.f;
#pragma unroll 2
                    for (int i = lane; i < (cn >> 2); i += 32) {
                        const float4 a = reinterpret_cast<const float4*>(rp)[i];
                        const float4 b = reinterpret_cast<const float4*>(xp)[i];
                        acc = fmaf(a.x, b.x, acc);
                        acc = fmaf(a.y, b.y, acc);
                        acc = fmaf(a.z, b.z, acc);
                        acc = fmaf(a.w, b.w, acc);
                    }
                    acc = warp_sum(acc);
                    if (lane == 0) s_part[warp] = acc;
                }
            }
            if (warp == nw - 1 && with_gate) {
                float acc = 0.f;
#pragma unroll 4
                for (int i = lane; i < H; i += 32) acc = fmaf(x32[i], ginp_s[i], acc);
                acc = warp_sum(acc);
                if (lane == 0) *s_sg = shared_sigmoid(acc);
            }
            __syncthreads();
            if (tid < nr) {
                const int spr = nwr / nr;
                float acc = 0.f;
                for (int q = 0; q < spr; ++q) acc += s_part[tid * spr + q];
                if (bias) acc = __fadd_rn(acc, bias[r0 + tid]);
                st_word_gpu(scores + r0 + tid, acc, tag);
            }
            if (tid >= nr && tid < r1 - r0) st_word_gpu(scores + r0 + tid, 0.f, tag);  // marker slots
            if (Is && !with_gate && tid == 0) *s_sg = 1.f;
        }
        // ---- the token quantised for the integer dot products
#pragma unroll 1
        for (int b = warp; b < H / 256; b += nw) quantize_block_ool(x32, sm + p.o_xq, H, b);
        __syncthreads();
        // router rows, gate vector and the token copy are consumed: the next
        // step's go out now
        if (tid == 0 && Ln) {
            issue_router(Ln);
            if (x_by_copy(s + 1)) issue_x(s + 1);
        }
        TRACE(3);

        // ---- warp 0: the routing (every CTA, identically) and the routed
        // copies; warps 1..: the shared expert's gate/up rows meanwhile
        if (warp == 0) {
            uint32_t sel_k = 0;
            int sel_id = 0;
            {
                uint32_t kk[8];
                int kid[8];
                if (!load_score_words(scores, E, S, tag, kWaitPolls,
                                      reinterpret_cast<uint32_t*>(s_scores), kk, kid) &&
                    lane == 0)
                    set_error(p.ctr, ST_TIMEOUT);
                topk_select_compact(kk, kid, K, sel_k, sel_id);
                if (lane < K) s_ids[lane] = sel_id;
            }
            __syncwarp();
            TRACE(4);
            // the selections this GPU holds, in top-k order
            const int e = lane < K ? s_ids[lane] : -1;
            const bool held = lane < K && e >= ebeg && e < ebeg + ecnt;
            const uint32_t hb = __ballot_sync(0xffffffffu, held);
            if (held) s_act[__popc(hb & ((1u << lane) - 1u))] = lane;
            const int A = __popc(hb);
            if (lane == 0) *s_nact = A;
            __syncwarp();
            // routed gate/up rows of [f0, f1) in chunks of CR rows (one
            // mbarrier each, in order, so compute starts on the first), lane
            // q issuing chunk q; the routed down rows (lane 16 + a: slot a)
            // at the same time
            const int f0 = part(A * I, c, G), f1 = part(A * I, c + 1, G);
            const int nrows = f1 - f0, CR = p.chunk_rows;
            const int nchunks = (nrows + CR - 1) / CR;
            if (lane < nchunks) {
                const int q = lane, q0 = q * CR, q1 = min(nrows, q0 + CR);
                mbar_arrive_expect_tx(&bars[3 + q], (uint32_t)((q1 - q0) * (rb_gate + rb_up)));
                for (int f = f0 + q0; f < f0 + q1;) {
                    const int a = f / I, r = f % I;
                    const int n = min(f0 + q1 - f, I - r);
                    const int64_t ex = s_ids[s_act[a]] - ebeg;
                    bulk_g2s(sm + p.o_rgate + (int64_t)(f - f0) * rb_gate, Ls->gate + ex * st_gate + r * rb_gate,
                             (uint32_t)(n * rb_gate), &bars[3 + q]);
                    bulk_g2s(sm + p.o_rup + (int64_t)(f - f0) * rb_up, Ls->up + ex * st_up + r * rb_up,
                             (uint32_t)(n * rb_up), &bars[3 + q]);
                    f += n;
                }
            }
            if (lane == 16) mbar_arrive_expect_tx(&bars[2], (uint32_t)(A * nh * rb_down));
            __syncwarp();
            if (lane >= 16 && lane - 16 < A && nh > 0) {
                const int a = lane - 16;
                const int64_t ex = s_ids[s_act[a]] - ebeg;
                bulk_g2s(sm + p.o_rdown + (int64_t)a * p.max_out_rows * rb_down,
                         Ls->down + ex * st_down + h0 * rb_down, (uint32_t)(nh * rb_down), &bars[2]);
            }
            // routing weights (float64 softmax over the selections), needed
            // only by the combine
            topk_weights_f32(sel_k, sel_id, K, s_ids, s_w);
            if (c == 0 && lane < K) {
                if (ids_out) ids_out[lane] = s_ids[lane];
                if (w_out) w_out[lane] = s_w[lane];
            }
        } else if (Is) {
            // shared expert gate/up (x is the token): warps 1.. while warp 0
            // routes; the activations go out as exchange words
            if (!mbar_wait(&bars[1], (ph >> 1) & 1u, kWaitPolls) && lane == 0) set_error(p.ctr, ST_TIMEOUT);
            const int rpw = 32 / lpr_h;
#pragma unroll 1
            for (int rb = (warp - 1) * rpw; rb < s1 - s0; rb += (nw - 1) * rpw) {
                const int rr = rb + sub_h;
                const bool ok = rr < s1 - s0;
                const int rs = ok ? rr : 0;
                const float2 gu = qdot2_rows<SGU>(L0.shared_gate_type, sm + p.o_sgate + rs * rb_sg,
                                                  L0.shared_up_type, sm + p.o_sup + rs * rb_su,
                                                  sm + p.o_xq, H, pr_h >> 2, pr_h & 3);
                const float g = group_sum(gu.x, lpr_h), u = group_sum(gu.y, lpr_h);
                if (ok && pr_h == 0) st_word_gpu(act_s + s0 + rr, (g * shared_sigmoid(g)) * u, tag);
            }
        }
        if (Is) ph ^= 2u;
        __syncthreads();
        // shared gate/up rows are consumed: the next step's go out now
        if (tid == 0 && Ln && Is) issue_sgu(Ln);
        TRACE(5);
        const int A = *s_nact;
        const int f0 = part(A * I, c, G), f1 = part(A * I, c + 1, G);
        const int nrows = f1 - f0;
        const int CR = p.chunk_rows;
        const int nchunks = (nrows + CR - 1) / CR;

        // ---- routed gate/up, chunk by chunk (one decoder call site for the
        // gate and the up row: the loops stay rolled so that the step's code
        // stays small in the instruction cache)
        {
            const int rpw = 32 / lpr_h;
            int waited = -1;
#pragma unroll 1
            for (int rb = warp * rpw; rb < nrows; rb += nw * rpw) {
                const int qlast = min(rb + rpw - 1, nrows - 1) / CR;
                while (waited < qlast) {
                    ++waited;
                    if (!mbar_wait(&bars[3 + waited], (ph >> (3 + waited)) & 1u, kWaitPolls) && lane == 0)
                        set_error(p.ctr, ST_TIMEOUT);
                    if (waited == 0) TRACE(6);
                }
                const int rr = rb + sub_h;
                const bool ok = rr < nrows;
                const int rs = ok ? rr : 0;
                const float2 gu = qdot2_rows<GU>(L0.gate_type, sm + p.o_rgate + rs * rb_gate, L0.up_type,
                                                 sm + p.o_rup + rs * rb_up, sm + p.o_xq, H, pr_h >> 2,
                                                 pr_h & 3);
                const float g = group_sum(gu.x, lpr_h), u = group_sum(gu.y, lpr_h);
                if (ok && pr_h == 0) {
                    const float sgm = 1.0f / (1.0f + expf(-g));
                    st_word_gpu(act_r + f0 + rr, (g * sgm) * u, tag);
                }
            }
            // every chunk barrier must have completed before the CTA moves on
            // (its copies write shared memory)
            for (int q = waited + 1; q < nchunks; ++q)
                if (!mbar_wait(&bars[3 + q], (ph >> (3 + q)) & 1u, kWaitPolls) && lane == 0)
                    set_error(p.ctr, ST_TIMEOUT);
            ph ^= ((1u << nchunks) - 1u) << 3;
        }
        TRACE(7);

        // ---- activations: every thread polls its share of the A*I routed
        // and Is shared exchange words (up to kGatherWords loads in flight),
        // then warp v quantises vector v (routed slots v < A, the shared one
        // v == A)
        float* act32 = reinterpret_cast<float*>(sm + p.o_act);
        const uint32_t qb = qvec_bytes(Imax);
        const int nvec = A + (Is ? 1 : 0);
        {
            const int nr_words = A * I, n_words = nr_words + Is;
            bool ok = true;
#pragma unroll 1
            for (int j0 = tid; j0 < n_words; j0 += kFusedThreads * kGatherWords) {
                uint32_t pend = 0;
                const uint64_t* srcw[kGatherWords];
                int dofs[kGatherWords];  // routed word j -> act32[(j / I) * Imax + j % I]
#pragma unroll
                for (int q = 0; q < kGatherWords; ++q) {
                    const int j = j0 + kFusedThreads * q;
                    if (j < n_words) pend |= 1u << q;
                    const int v = j < nr_words ? j / I : A;
                    srcw[q] = j < nr_words ? act_r + j : act_s + (j - nr_words);
                    dofs[q] = v * Imax + (j < nr_words ? j - v * I : j - nr_words);
                }
                for (uint32_t round = 0; pend != 0u; ++round) {
                    if (round == kWaitPolls) {
                        ok = false;
                        break;
                    }
                    uint64_t wv[kGatherWords];
#pragma unroll
                    for (int q = 0; q < kGatherWords; ++q) wv[q] = ((pend >> q) & 1u) ? ld_word_gpu(srcw[q]) : 0ull;
#pragma unroll
                    for (int q = 0; q < kGatherWords; ++q) {
                        if (((pend >> q) & 1u) && (uint32_t)(wv[q] >> 32) == tag) {
                            pend &= ~(1u << q);
                            act32[dofs[q]] = __uint_as_float((uint32_t)wv[q]);
                        }
                    }
                }
            }
            if (!ok) set_error(p.ctr, ST_TIMEOUT);
        }
        __syncthreads();
        TRACE(8);
        for (int v = warp; v < nvec; v += nw) {
            const int n = v < A ? I : Is;
#pragma unroll 1
            for (int b = 0; b < n / 256; ++b) quantize_block_ool(act32 + v * Imax, sm + p.o_aq + v * qb, n, b);
        }
        __syncthreads();
        TRACE(9);
        // the routed and shared down rows of this CTA
        if (tid == 0 && !mbar_wait(&bars[2], (ph >> 2) & 1u, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
        ph ^= 4u;
        if (Is) {
            if (tid == 0 && !mbar_wait(&bars[kSdBar], (ph >> kSdBar) & 1u, kWaitPolls)) set_error(p.ctr, ST_TIMEOUT);
            ph ^= 1u << kSdBar;
        }
        __syncthreads();
        TRACE(10);

        // ---- down rows [h0, h1) of every vector: item = (vector, pair of
        // row groups), the activation codes loaded once per item; the shared
        // vector's row groups first, one per item
        {
            const int rpw_i = 32 / p.lpr_i, rpw_s = 32 / p.lpr_is;
            const int ng_i = (nh + rpw_i - 1) / rpw_i, ng_s = Is ? (nh + rpw_s - 1) / rpw_s : 0;
            const int np_i = (ng_i + 1) / 2, np_s = ng_s;
#pragma unroll 1
            for (int it = warp; it < A * np_i + np_s; it += nw) {
                const bool sh = it < np_s;
                const int v = sh ? A : (it - np_s) / np_i;
                const int gp = sh ? it : (it - np_s) % np_i;
                const int lpr = sh ? p.lpr_is : p.lpr_i;
                const int rpw = 32 / lpr, sub = lane / lpr, pr = lane % lpr;
                const int type = sh ? L0.shared_down_type : L0.down_type;
                const int64_t rb = sh ? rb_sd : rb_down;
                const uint8_t* rows = sh ? sm + p.o_sdown : sm + p.o_rdown + (int64_t)v * p.max_out_rows * rb_down;
                const int n = sh ? Is : I;
                uint8_t* codes = sm + p.o_aq + v * qb;
                if (sh) {
                    const int rr = gp * rpw + sub;
                    const bool ok = rr < nh;
                    float d = qdot1_row<SDN>(type, rows + (ok ? rr : 0) * rb, codes, n, pr >> 2, pr & 3);
                    d = group_sum(d, lpr);
                    if (ok && pr == 0) s_vout[v * p.max_out_rows + rr] = d;
                } else {
                    const int ra = 2 * gp * rpw + sub, rb2 = ra + rpw;
                    const bool oka = ra < nh, okb = rb2 < nh;
                    const float2 d = qdot2_rows<DN>(type, rows + (oka ? ra : 0) * rb, type,
                                                    rows + (okb ? rb2 : 0) * rb, codes, n, pr >> 2, pr & 3);
                    const float da = group_sum(d.x, lpr), db = group_sum(d.y, lpr);
                    if (pr == 0) {
                        if (oka) s_vout[v * p.max_out_rows + ra] = da;
                        if (okb) s_vout[v * p.max_out_rows + rb2] = db;
                    }
                }
            }
        }
        __syncthreads();
        // shared down rows are consumed: the next step's go out now
        if (tid == 0 && Ln && Is) issue_sdown(Ln);
        TRACE(11);
        // ---- weighted sum in top-k order, + shared (moe_layer.py:85-86, 102-105);
        // block steps add the residual h to the binary16-rounded MoE output
        // (transformer.py:192-204, 229-247).  A chained next step reads the
        // rows as exchange words.
        {
            uint64_t* ywn = p.yw + (size_t)buf * H;
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
                if (next_chains) st_word_gpu(ywn + h0 + rr, comb, tag);
                if (yout) yout[h0 + rr] = comb;
            }
        }
        __syncthreads();
        TRACE(12);
#undef TRACE
    }
    // ---- exit: the last CTA advances the sequence word for the next launch
    // With a host-visible error word (the synchronous host-buffer call) the
    // word is also the completion signal the host waits on: every CTA's
    // writes to host memory are ordered before its exit count at system
    // scope, and the last CTA releases the word after seeing every count.
    if (tid == 0) {
        if (p.err_out) __threadfence_system();
        else __threadfence();
        const uint32_t t = atomicAdd(p.ctr + C_EXIT, 1u);
        if (t == (uint32_t)G - 1) {
            p.ctr[C_EXIT] = 0;
            p.ctr[C_SEQ] = seq0 + (uint32_t)p.n_steps;
            if (p.err_out) {
                const int err = atomicExch(reinterpret_cast<int*>(p.ctr + C_ERROR), 0);
                __threadfence_system();
                st_release_sys(reinterpret_cast<uint32_t*>(p.err_out), (uint32_t)err);
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

static bool fused_plan(const moe_b200_layer* L, bool shared, int G, FusedParams& p);

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
    FusedParams p;
    return fused_plan(L, shared, sm_count(), p);
}

size_t fused_workspace_bytes(const moe_b200_layer* L) {
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate : L->intermediate;
    const int S = L->n_experts > sm_count() ? L->n_experts : sm_count();
    // counters, then two buffers (step parity) of score slots, routed and
    // shared activations and the layer output words
    return 256 + align_up((size_t)2 * S * 8) + align_up((size_t)2 * L->top_k * L->intermediate * 8) +
           align_up((size_t)2 * Imax * 8) + align_up((size_t)2 * L->hidden * 8);
}

static bool fused_plan(const moe_b200_layer* L, bool shared, int G, FusedParams& p) {
    const int H = L->hidden, I = L->intermediate, E = L->n_experts, K = L->top_k;
    const int Is = shared ? L->shared_intermediate : 0;
    const int Imax = Is > I ? Is : I;
    p.G = G;
    p.S = E > G ? E : G;
    p.with_shared = shared ? 1 : 0;
    p.max_router_rows = (p.S + G - 1) / G;
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
    p.o_ginp = take(Is ? (uint64_t)H * 4 : 0);
    p.o_sgate = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_gate_type, H) : 0);
    p.o_sup = take(Is ? (uint64_t)p.max_sgu_rows * row_bytes(L->shared_up_type, H) : 0);
    p.o_sdown = take(Is ? (uint64_t)p.max_out_rows * row_bytes(L->shared_down_type, Is) : 0);
    p.o_rgate = take((uint64_t)p.max_rgu_rows * row_bytes(L->gate_type, H));
    p.o_rup = take((uint64_t)p.max_rgu_rows * row_bytes(L->up_type, H));
    p.o_rdown = take((uint64_t)K * p.max_out_rows * row_bytes(L->down_type, I));
    p.o_act = take((uint64_t)(K + 1) * Imax * 4);
    p.o_aq = take((uint64_t)(K + 1) * qvec_bytes(Imax));
    p.o_misc = take(512 + ((5 * p.S + 15) & ~15) + (uint64_t)(K + 1) * p.max_out_rows * 4);
    p.total = o;
    // one warp-level top-k over at most 256 score slots; the router rows of
    // a CTA fit one pass of all warps but one
    if (p.S > 256 || p.max_router_rows > kFusedThreads / 32 - 1) return false;
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
    off += align_up((size_t)2 * p.S * 8);
    p.act_r = reinterpret_cast<uint64_t*>(base + off);
    off += align_up((size_t)2 * L->top_k * L->intermediate * 8);
    p.act_s = reinterpret_cast<uint64_t*>(base + off);
    off += align_up((size_t)2 * Imax * 8);
    p.yw = reinterpret_cast<uint64_t*>(base + off);
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
