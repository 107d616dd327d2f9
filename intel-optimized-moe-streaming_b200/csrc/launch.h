// launch.h -- internal launchers shared by the translation units.
#pragma once

#include "common.cuh"
#include "moe_b200.h"

// This rank's expert-parallel exchange buffer and its peers' mappings
// (decode_multi.cu).  Region offsets are the same on every rank.
struct moe_b200_ep {
    int world = 0, rank = 0, tq = 0, H = 0, G = 0, dev = 0;
    char* local = nullptr;    // this rank's buffer
    char* peer[8] = {};       // every rank's buffer in this process (peer[rank] = local)
    size_t o_xs = 0, o_yp = 0, o_seq = 0, bytes = 0;
    bool connected = false;
};

namespace moeb200 {

int sm_count();  // multiprocessors of the current device (cached per device)

// Lays out regions (256-byte aligned) inside one buffer.
struct Stager {
    size_t used = 0;
    size_t take(size_t bytes) {
        const size_t at = used;
        used += align_up(bytes);
        return at;
    }
};

cudaError_t launch_dequant(int type, const void* src, void* dst, int64_t n, bool f16,
                           cudaStream_t stream);

// One DeltaNet step (cpp/moe_delta.cpp:18-69), all pointers on the device.
// decay: per-head exp(gate) computed by the caller, or null to compute it on
// the device from gate.  bad: null, or a word the kernel lowers (atomicMin)
// to the flat index h * dv + r of every row whose output is not finite.
struct DeltaArgs {
    float* state;          // [heads][dv][dk], updated in place
    const float* q;        // [heads][dk]
    const float* k;        // [heads][dk]
    const float* v;        // [heads][dv]
    const float* beta;     // [heads]
    const float* gate;     // [heads]
    const double* decay;   // [heads] or null
    float* out;            // [heads][dv]
    unsigned* bad;
    unsigned* err;         // null, or a word set to 1 when a bounded wait gave up
    int heads, dk, dv;
};
cudaError_t launch_delta_heads(const DeltaArgs& a, cudaStream_t stream);
// moe_delta_heads with every array in (pageable) host memory: pinned staging
// and a chunked copy/compute pipeline (delta_host.cu).  Returns 0, -2 (the
// reference's early stop) or ST_INTERNAL with *ce set.
int delta_heads_host(float* state, const float* q, const float* k, const float* v,
                     const float* beta, const float* gate, float* output, int heads, int dk,
                     int dv, cudaError_t* ce);

// memcpy split over a few persistent host threads (hostcopy.cu); small copies
// run on the calling thread.
void host_parallel_copy(void* dst, const void* src, size_t bytes);

// Routing of T tokens: fp32 scores [T x E] (+ bias), top-K ids/weights, and
// the shared-expert gate sigmoid(x . gate_inp) per token.
struct RoutePlan {
    int T, E, K, H;
    const float* x;          // [T x H]
    const float* router;     // [E x H]
    const float* bias;       // [E] or null
    const float* gate_inp;   // [H] or null (no shared expert)
    float* scores;           // [T x E]
    int32_t* ids;            // [T x K]
    float* w;                // [T x K]
    float* sg;               // [T]
};
cudaError_t launch_route(const RoutePlan& p, cudaStream_t stream);

// Expert work of T tokens with K routed slots each (+ the shared expert),
// computed by the exact engine: every weight dequantised bit-exactly, fp32
// fused multiply-add accumulation.
struct ExactPlan {
    int T, K, H, I, Is, Imax;
    int round16;             // fp16_graph rounding points on routed experts
    int expert_begin;        // global id of the first held expert
    int expert_count;
    const float* x;          // [T x H]
    const int32_t* ids;      // [T x K] global expert ids, or null (expert 0)
    const float* w;          // [T x K] routing weights, or null (1.0)
    const float* sg;         // [T] shared gate, null without shared expert
    QMat gate, up, down;
    QMat sgate, sup, sdown;  // base null without shared expert
    float* act;              // [T x (K+1) x Imax]
    float* y;                // [T x H]
};
cudaError_t launch_exact(const ExactPlan& p, cudaStream_t stream);

// Fused single-token layer decode (decode.cu).  The first 256 bytes of the
// workspace hold its counters and error word (zero before the first launch;
// the kernel leaves them zero).
bool fused_supported(const moe_b200_layer* L, int T, int flags);
size_t fused_workspace_bytes(const moe_b200_layer* L);
cudaError_t launch_decode_fused(const moe_b200_layer* L, int flags, const float* x, float* y,
                                int32_t* ids_out, float* w_out, void* ws, cudaStream_t stream,
                                bool* launched);
// n_steps single-token steps from device tables in one launch (every layer
// shares L0's shapes and block formats; L0's flags apply to all).
// Single-token fused decode for host buffers the device can read and write
// (pinned): a graph of a copy kernel (x_host -> x_stage, device staging
// rows) and the fused kernel, which writes y, the routing and the error word
// (err_host, cleared on the device) straight to host memory.
cudaError_t launch_decode_fused_host(const moe_b200_layer* L, int flags, const float* x_host,
                                     float* x_stage, float* y_host, int32_t* ids_host,
                                     float* w_host, int* err_host, void* ws, cudaStream_t stream,
                                     bool* launched);
cudaError_t launch_decode_steps(const moe_b200_layer* L0, const moe_b200_layer* layers,
                                const moe_b200_step* steps, int n_steps, float eps, void* ws,
                                cudaStream_t stream, bool* launched);
// Fused layer decode of 1..8 tokens (decode_multi.cu); the shared expert
// goes to tokens [sh_lo, sh_hi) only (with_shared layers).  Shares the
// counter words of the single-token kernel.
bool multi_supported(const moe_b200_layer* L, int T, int flags);
size_t multi_workspace_bytes(const moe_b200_layer* L, int T);
// With an exchange context xc (expert-parallel over peer memory): x and y
// are this rank's xc->tq tokens, T = world * tq, the shared expert covers
// the own tokens and the routing outputs all T gathered tokens.
cudaError_t launch_decode_multi(const moe_b200_layer* L, int flags, const float* x, int T,
                                int sh_lo, int sh_hi, float* y, int32_t* ids_out, float* w_out,
                                void* ws, cudaStream_t stream, bool* launched,
                                const moe_b200_ep* xc = nullptr);
int ep_create(int world, int rank, int tq, int H, moe_b200_ep** out, void* blob_out,
              cudaError_t* ce);
int ep_connect(moe_b200_ep* c, const void* blobs, cudaError_t* ce);
void ep_destroy(moe_b200_ep* c);
void set_fused_trace(void* buf, int capacity_ctas);
uint64_t* trace_buffer(int* capacity_ctas);  // the buffer set above (this thread)

// Many-token layer on the tcgen05 tensor cores (prefill.cu).  x is fp32 or
// (x_bf16) bf16 [T x H]; y is written in full.
bool prefill_supported(const moe_b200_layer* L, int flags);
size_t prefill_workspace_bytes(const moe_b200_layer* L, int T);
int prefill_run(const moe_b200_layer* L, const void* x, int x_bf16, int T, float* y,
                int32_t* ids_out, float* w_out, void* ws, size_t ws_bytes, cudaStream_t s,
                cudaError_t* ce);
int prefill_kernels(const moe_b200_layer* L, int T);

// Identity-mixer transformer block around a many-token MoE call (block.cu).
cudaError_t launch_block_prepare(const float* x, float* h, float* n, int T, int H, float eps,
                                 cudaStream_t s);
cudaError_t launch_block_finish(const float* h, const float* m, float* y, int T, int H,
                                cudaStream_t s);

}  // namespace moeb200
