// noalloc.cu -- a single-expert entry point that allocates nothing.
//
// Some callers cannot call cudaMalloc: a serving process that reserved all
// device memory up front for its own pool, or a thread that must not enter
// the CUDA allocator while other work is in flight (cudaFree, and a
// cudaMalloc that has to return memory first, synchronise the whole
// device).  moe_b200_expert_noalloc gives them the exact-engine SwiGLU
// expert with its scratch -- the intermediate activations -- in the
// file-scope array below instead of in allocated memory.  The caller still
// passes inputs and outputs (device memory).
//
// The array lives in every GPU that loads this library until the process
// exits.  All calls on a GPU share it and it keeps the last call's
// contents; nothing in it needs to start at zero (every activation a call
// reads, it first writes).  Calls whose kernels overlap on the GPU (two
// streams, two threads) race on it: order them on one stream.
#include <mutex>

#include "launch.h"

namespace moeb200 {

constexpr int kNoAllocMaxInter = MOE_B200_NOALLOC_MAX_INTERMEDIATE;

// Activations of one call: slot 0 (the expert) and slot 1 (the exact
// engine's shared-expert slot, unused here), kNoAllocMaxInter floats each.
static __device__ __align__(256) float g_noalloc_act[2 * kNoAllocMaxInter];

static std::mutex g_noalloc_mu;
static float* g_noalloc_ptr[64] = {};

// Device address of g_noalloc_act on the current device.  The host-side
// name of the array is only a stand-in; the address comes from
// cudaGetSymbolAddress, once per device, with that device current.
static cudaError_t noalloc_scratch(float** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_act);
        if (e != cudaSuccess) return e;
        g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    *out = g_noalloc_ptr[dev];
    return cudaSuccess;
}

static bool device_ptr(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

}  // namespace moeb200

using namespace moeb200;

extern "C" int moe_b200_expert_noalloc(int gate_type, const uint8_t* gate, int64_t gate_bytes,
                                       int up_type, const uint8_t* up, int64_t up_bytes,
                                       int down_type, const uint8_t* down, int64_t down_bytes,
                                       const float* input, int hidden, int intermediate,
                                       float* output, int fp16_graph, void* stream) {
    const int types[3] = {gate_type, up_type, down_type};
    const int cols[3] = {hidden, hidden, intermediate};
    const int rows[3] = {intermediate, intermediate, hidden};
    const int64_t sizes[3] = {gate_bytes, up_bytes, down_bytes};
    if (!gate || !up || !down || !input || !output || hidden <= 0 || intermediate <= 0 ||
        hidden > 65536 || intermediate > kNoAllocMaxInter || (fp16_graph != 0 && fp16_graph != 1))
        return ST_ARG;
    for (int i = 0; i < 3; ++i) {
        const int bs = block_size(types[i]);
        if (!bs || cols[i] % bs) return ST_TYPE;
        if (sizes[i] != (int64_t)rows[i] * (cols[i] / bs) * block_bytes(types[i])) return ST_BYTES;
    }
    const void* ptrs[5] = {gate, up, down, input, output};
    for (const void* p : ptrs)
        if (!device_ptr(p)) return ST_ARG;
    if (((uintptr_t)input | (uintptr_t)output) & 15u) return ST_ALIGN;
    float* act = nullptr;
    cudaError_t e = noalloc_scratch(&act);
    if (e != cudaSuccess) return ST_CUDA;
    ExactPlan p{};
    p.T = 1;
    p.K = 1;
    p.H = hidden;
    p.I = intermediate;
    p.Is = 0;
    p.Imax = intermediate;
    p.round16 = fp16_graph;
    p.expert_begin = 0;
    p.expert_count = 1;
    p.x = input;
    p.gate.base = gate;
    p.gate.type = gate_type;
    p.gate.rows = intermediate;
    p.gate.cols = hidden;
    p.gate.row_bytes = row_bytes(gate_type, hidden);
    p.gate.stride = gate_bytes;
    p.up.base = up;
    p.up.type = up_type;
    p.up.rows = intermediate;
    p.up.cols = hidden;
    p.up.row_bytes = row_bytes(up_type, hidden);
    p.up.stride = up_bytes;
    p.down.base = down;
    p.down.type = down_type;
    p.down.rows = hidden;
    p.down.cols = intermediate;
    p.down.row_bytes = row_bytes(down_type, intermediate);
    p.down.stride = down_bytes;
    p.act = act;
    p.y = output;
    e = launch_exact(p, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ST_OK : ST_CUDA;
}
