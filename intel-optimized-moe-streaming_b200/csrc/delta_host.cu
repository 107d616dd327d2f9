// moe_delta_heads for host arrays (the reference caller's numpy state): the
// state crosses PCIe in and out every call, so the call is a pipeline over
// head chunks.  Per chunk: a parallel host copy into pinned staging, one
// host-to-device copy and the step kernel on stream s0; the device-to-host
// copy of the chunk's state, outputs and status word on stream s1, so the
// copy engines move chunk i back while chunk i+1 goes in; the host copies
// chunk i out of pinned staging as soon as it has landed.  The reference's
// early stop (cpp/moe_delta.cpp:64-67) is kept: the first chunk whose status
// word names a non-finite row is copied out only up to that row (state) and
// before it (outputs), and no later chunk is copied out.
#include <cmath>
#include <cstring>

#include "launch.h"

namespace moeb200 {

namespace {

constexpr int kMaxChunks = 4;

struct DeltaHostStage {
    int device = -1;
    cudaStream_t s0 = nullptr, s1 = nullptr;
    cudaEvent_t run[kMaxChunks] = {}, back[kMaxChunks] = {};
    char* pinned = nullptr;
    char* dev = nullptr;
    size_t cap = 0;

    cudaError_t ensure(size_t bytes) {
        cudaError_t e = cudaSuccess;
        if (!s0) {
            e = cudaStreamCreateWithFlags(&s0, cudaStreamNonBlocking);
            if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s1, cudaStreamNonBlocking);
            for (int i = 0; i < kMaxChunks && e == cudaSuccess; ++i) {
                e = cudaEventCreateWithFlags(&run[i], cudaEventDisableTiming);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&back[i], cudaEventDisableTiming);
            }
            if (e != cudaSuccess) return e;
        }
        if (bytes <= cap) return cudaSuccess;
        if (pinned) cudaFreeHost(pinned);
        if (dev) cudaFree(dev);
        pinned = dev = nullptr;
        cap = 0;
        const size_t want = align_up(bytes + bytes / 4);
        e = cudaHostAlloc(reinterpret_cast<void**>(&pinned), want, cudaHostAllocDefault);
        if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&dev), want);
        if (e != cudaSuccess) return e;
        cap = want;
        return cudaSuccess;
    }
};

DeltaHostStage* stage_for_device() {
    static thread_local DeltaHostStage per_device[16];
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess || d < 0 || d >= 16) return nullptr;
    per_device[d].device = d;
    return &per_device[d];
}

}  // namespace

int delta_heads_host(float* state, const float* q, const float* k, const float* v,
                     const float* beta, const float* gate, float* output, int heads, int dk,
                     int dv, cudaError_t* ce) {
    *ce = cudaSuccess;
    DeltaHostStage* sg = stage_for_device();
    if (!sg) {
        *ce = cudaErrorInvalidDevice;
        return ST_INTERNAL;
    }
    const size_t rows = (size_t)heads * dv;
    const size_t row_bytes = (size_t)dk * 4;
    // pinned and device buffers share one layout
    Stager st;
    const size_t o_bad = st.take(kMaxChunks * 4);   // per chunk: first non-finite row
    const size_t o_err = st.take(4);                 // a bounded device wait gave up
    const size_t o_out = st.take(rows * 4);
    const size_t o_decay = st.take((size_t)heads * 8);   // start of the inputs region
    const size_t o_beta = st.take((size_t)heads * 4);
    const size_t o_v = st.take(rows * 4);
    const size_t o_q = st.take((size_t)heads * row_bytes);
    const size_t o_k = st.take((size_t)heads * row_bytes);
    const size_t o_state = st.take(rows * row_bytes);
    cudaError_t e = sg->ensure(st.used);
    if (e != cudaSuccess) {
        *ce = e;
        return ST_INTERNAL;
    }
    char* P = sg->pinned;
    char* D = sg->dev;
    // small inputs; decay = exp(double(gate)) with the host libm, as the
    // reference computes it
    double* decay = reinterpret_cast<double*>(P + o_decay);
    for (int h = 0; h < heads; ++h) decay[h] = std::exp(static_cast<double>(gate[h]));
    std::memcpy(P + o_beta, beta, (size_t)heads * 4);
    std::memcpy(P + o_v, v, rows * 4);
    host_parallel_copy(P + o_q, q, (size_t)heads * row_bytes);
    host_parallel_copy(P + o_k, k, (size_t)heads * row_bytes);
    e = cudaMemcpyAsync(D + o_decay, P + o_decay, o_state - o_decay, cudaMemcpyHostToDevice, sg->s0);
    if (e == cudaSuccess) e = cudaMemsetAsync(D + o_bad, 0xFF, kMaxChunks * 4, sg->s0);
    if (e == cudaSuccess) e = cudaMemsetAsync(D + o_err, 0, 4, sg->s0);

    const int chunks = heads < kMaxChunks ? heads : kMaxChunks;
    const int per = (heads + chunks - 1) / chunks;
    int launched = 0;
    for (int c = 0; c < chunks && e == cudaSuccess; ++c) {
        const int h0 = c * per;
        const int hc = (h0 + per <= heads ? per : heads - h0);
        if (hc <= 0) break;
        const size_t r0 = (size_t)h0 * dv, rc = (size_t)hc * dv;
        host_parallel_copy(P + o_state + r0 * row_bytes, state + r0 * dk, rc * row_bytes);
        e = cudaMemcpyAsync(D + o_state + r0 * row_bytes, P + o_state + r0 * row_bytes,
                            rc * row_bytes, cudaMemcpyHostToDevice, sg->s0);
        if (e != cudaSuccess) break;
        DeltaArgs a{};
        a.state = reinterpret_cast<float*>(D + o_state) + r0 * dk;
        a.q = reinterpret_cast<const float*>(D + o_q) + (size_t)h0 * dk;
        a.k = reinterpret_cast<const float*>(D + o_k) + (size_t)h0 * dk;
        a.v = reinterpret_cast<const float*>(D + o_v) + r0;
        a.beta = reinterpret_cast<const float*>(D + o_beta) + h0;
        a.gate = nullptr;
        a.decay = reinterpret_cast<const double*>(D + o_decay) + h0;
        a.out = reinterpret_cast<float*>(D + o_out) + r0;
        a.bad = reinterpret_cast<unsigned*>(D + o_bad) + c;
        a.err = reinterpret_cast<unsigned*>(D + o_err);
        a.heads = hc;
        a.dk = dk;
        a.dv = dv;
        e = launch_delta_heads(a, sg->s0);
        if (e == cudaSuccess) e = cudaEventRecord(sg->run[c], sg->s0);
        if (e == cudaSuccess) e = cudaStreamWaitEvent(sg->s1, sg->run[c], 0);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(P + o_state + r0 * row_bytes, D + o_state + r0 * row_bytes,
                                rc * row_bytes, cudaMemcpyDeviceToHost, sg->s1);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(P + o_out + r0 * 4, D + o_out + r0 * 4, rc * 4,
                                cudaMemcpyDeviceToHost, sg->s1);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(P + o_bad + c * 4, D + o_bad + c * 4, 4, cudaMemcpyDeviceToHost,
                                sg->s1);
        if (e == cudaSuccess)
            e = cudaMemcpyAsync(P + o_err, D + o_err, 4, cudaMemcpyDeviceToHost, sg->s1);
        if (e == cudaSuccess) e = cudaEventRecord(sg->back[c], sg->s1);
        if (e == cudaSuccess) ++launched;
    }
    int status = ST_OK;
    for (int c = 0; c < launched && e == cudaSuccess && status == ST_OK; ++c) {
        e = cudaEventSynchronize(sg->back[c]);
        if (e != cudaSuccess) break;
        const size_t r0 = (size_t)c * per * dv;
        const size_t rc = (size_t)((c + 1) * per <= heads ? per : heads - c * per) * dv;
        if (*reinterpret_cast<const unsigned*>(P + o_err)) {
            status = ST_TIMEOUT;
            break;
        }
        const unsigned bad = reinterpret_cast<const unsigned*>(P + o_bad)[c];
        size_t n_state = rc, n_out = rc;
        if (bad != 0xFFFFFFFFu) {
            n_state = (size_t)bad + 1;
            n_out = bad;
            status = -2;   // cpp/moe_delta.cpp:66
        }
        host_parallel_copy(state + r0 * dk, P + o_state + r0 * row_bytes, n_state * row_bytes);
        std::memcpy(output + r0, P + o_out + r0 * 4, n_out * 4);
    }
    // nothing may still read or write the staging when the call returns
    const cudaError_t e0 = cudaStreamSynchronize(sg->s0);
    const cudaError_t e1 = cudaStreamSynchronize(sg->s1);
    if (e == cudaSuccess) e = e0 != cudaSuccess ? e0 : e1;
    if (e != cudaSuccess) {
        *ce = e;
        return ST_INTERNAL;
    }
    return status;
}

}  // namespace moeb200
