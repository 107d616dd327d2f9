// abi.cu -- the extern "C" entry points of libmoe_b200.so (include/moe_b200.h).
//
// Reference-compatible exports accept host or device pointers.  Host buffers
// are copied through a per-thread, per-device scratch allocation on a
// per-thread stream, so concurrent callers (the reference fans experts out
// over a ThreadPoolExecutor, src/flash_moe/moe_layer.py:76-97) never share
// device state and each call is deterministic.
#include <chrono>
#include <cmath>
#include <cstring>
#include <new>
#include <vector>

#include "launch.h"

namespace moeb200 {

static thread_local int tl_last_cuda = 0;

static int fail(cudaError_t e, int code) {
    tl_last_cuda = (int)e;
    return code;
}

int sm_count() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

static inline size_t align256(size_t v) { return align_up(v); }

// Per-thread scratch on one device: a stream and a growable device buffer.
struct Scratch {
    int device = -1;
    cudaStream_t stream = nullptr;
    void* buf = nullptr;
    size_t cap = 0;
    void* host = nullptr;  // pinned staging for results read on the host
    size_t hcap = 0;

    cudaError_t ensure_host(size_t bytes) {
        if (bytes <= hcap) return cudaSuccess;
        if (host) cudaFreeHost(host);
        host = nullptr;
        hcap = 0;
        const size_t want = align256(bytes);
        cudaError_t e = cudaMallocHost(&host, want);
        if (e != cudaSuccess) return e;
        hcap = want;
        return cudaSuccess;
    }

    cudaError_t ensure(size_t bytes) {
        if (!stream) {
            cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
            if (e != cudaSuccess) return e;
        }
        if (bytes <= cap) return cudaSuccess;
        if (buf) cudaFree(buf);
        buf = nullptr;
        cap = 0;
        const size_t want = align256(bytes + bytes / 4);
        cudaError_t e = cudaMalloc(&buf, want);
        if (e != cudaSuccess) return e;
        cap = want;
        return cudaSuccess;
    }
    ~Scratch() {
        if (device < 0) return;
        int prev = 0;
        if (cudaGetDevice(&prev) != cudaSuccess) return;
        cudaSetDevice(device);
        if (buf) cudaFree(buf);
        if (host) cudaFreeHost(host);
        if (stream) cudaStreamDestroy(stream);
        cudaSetDevice(prev);
    }
};

static Scratch* thread_scratch() {
    static thread_local Scratch per_device[16];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 16) return nullptr;
    per_device[dev].device = dev;
    return &per_device[dev];
}

// true when p is device (or managed) memory the GPU can use in place.
static bool on_device(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

// true when p is device (or managed) memory of the current device.
static bool on_this_device(const void* p) {
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) && a.device == dev;
}

// moe_quant_expert's output rule on the device: the rows of y up to and
// including the first non-finite one (all rows when every one is finite)
// go to out; res[0] = that row count, res[1] = 1 when a row was non-finite.
__global__ void __launch_bounds__(256) k_emit_rows(const float* y, float* out, int n, int* res) {
    __shared__ int s_first;
    if (threadIdx.x == 0) s_first = n;
    __syncthreads();
    int first = n;
    for (int r = threadIdx.x; r < n; r += blockDim.x)
        if (!isfinite(y[r])) {
            first = r;
            break;
        }
    atomicMin(&s_first, first);
    __syncthreads();
    const int m = s_first < n ? s_first + 1 : n;
    for (int r = threadIdx.x; r < m; r += blockDim.x) out[r] = y[r];
    if (threadIdx.x == 0) {
        res[0] = m;
        res[1] = s_first < n ? 1 : 0;
    }
}

static int check_qmat(int type, const void* base, int rows, int cols) {
    if (!supported(type) || cols % block_size(type)) return ST_TYPE;
    if (!base) return ST_ARG;
    if (!aligned16(base)) return ST_ALIGN;
    (void)rows;
    return ST_OK;
}

static QMat qmat(int type, const void* base, int rows, int cols) {
    QMat m;
    m.base = static_cast<const uint8_t*>(base);
    m.type = type;
    m.rows = rows;
    m.cols = cols;
    m.row_bytes = row_bytes(type, cols);
    m.stride = m.row_bytes * rows;
    return m;
}

static int check_layer(const moe_b200_layer* L) {
    if (!L) return ST_ARG;
    if (L->hidden <= 0 || L->intermediate <= 0 || L->hidden > 65536 || L->intermediate > 65536)
        return ST_ARG;
    if (L->n_experts < 1 || L->top_k < 1 || L->top_k > 16 || L->top_k > L->n_experts) return ST_ARG;
    if (L->expert_begin < 0 || L->expert_count < 1 ||
        L->expert_begin + L->expert_count > L->n_experts)
        return ST_ARG;
    if (!L->router || !aligned16(L->router)) return L->router ? ST_ALIGN : ST_ARG;
    int st;
    if ((st = check_qmat(L->gate_type, L->gate, L->intermediate, L->hidden)) != ST_OK) return st;
    if ((st = check_qmat(L->up_type, L->up, L->intermediate, L->hidden)) != ST_OK) return st;
    if ((st = check_qmat(L->down_type, L->down, L->hidden, L->intermediate)) != ST_OK) return st;
    if (L->shared_intermediate < 0 || L->shared_intermediate > 65536) return ST_ARG;
    if (L->shared_intermediate > 0) {
        const int Is = L->shared_intermediate;
        if ((st = check_qmat(L->shared_gate_type, L->shared_gate, Is, L->hidden)) != ST_OK) return st;
        if ((st = check_qmat(L->shared_up_type, L->shared_up, Is, L->hidden)) != ST_OK) return st;
        if ((st = check_qmat(L->shared_down_type, L->shared_down, L->hidden, Is)) != ST_OK) return st;
        if (!L->shared_gate_inp) return ST_ARG;
    }
    return ST_OK;
}

// Workspace regions of one decode call.
struct DecodeWs {
    size_t scores, ids, w, sg, act, total;
};

static DecodeWs decode_ws(const moe_b200_layer* L, int T) {
    const int Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate
                                                              : L->intermediate;
    Stager s;
    s.used = 256;  // counters and error word of the fused kernel
    DecodeWs w;
    w.scores = s.take((size_t)T * L->n_experts * 4);
    w.ids = s.take((size_t)T * L->top_k * 4);
    w.w = s.take((size_t)T * L->top_k * 4);
    w.sg = s.take((size_t)T * 4);
    w.act = s.take((size_t)T * (L->top_k + 1) * Imax * 4);
    w.total = s.used;
    const size_t fused = fused_workspace_bytes(L);
    if (fused > w.total) w.total = fused;
    const size_t multi = multi_workspace_bytes(L, T);
    if (multi > w.total) w.total = multi;
    return w;
}

}  // namespace moeb200

using namespace moeb200;

extern "C" {

int moe_b200_version(void) { return 100; }

int moe_b200_workspace_init(void* workspace, size_t workspace_bytes, void* stream) {
    if (!workspace || workspace_bytes < 256) return ST_ARG;
    cudaError_t e = cudaMemsetAsync(workspace, 0, workspace_bytes, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_workspace_error(void* workspace, void* stream, int* error) {
    if (!workspace || !error) return ST_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int* word = reinterpret_cast<int*>(static_cast<char*>(workspace) + 32);
    cudaError_t e = cudaMemcpyAsync(error, word, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e == cudaSuccess && *error != 0) e = cudaMemsetAsync(word, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_last_cuda_error(void) { return tl_last_cuda; }

int moe_b200_set_trace(void* device_buffer, int capacity_ctas) {
    if (device_buffer && capacity_ctas < 1) return ST_ARG;
    set_fused_trace(device_buffer, device_buffer ? capacity_ctas : 0);
    return ST_OK;
}

int dequant_k_supported(int type) { return supported(type) ? 1 : 0; }

int dequant_k_block_size(int type) { return block_size(type); }

int dequant_k(int type, const uint8_t* src, void* dst, int64_t n, int want_f16) {
    const int bs = block_size(type);
    if (bs == 0 || src == nullptr || dst == nullptr) return ST_ARG;
    if (n <= 0 || n % bs != 0) return ST_ARG;
    Scratch* sc = thread_scratch();
    if (!sc) return fail(cudaErrorInvalidDevice, ST_CUDA);
    const size_t in_bytes = (size_t)(n / bs) * block_bytes(type);
    const size_t out_bytes = (size_t)n * (want_f16 ? 2 : 4);
    const bool src_dev = on_device(src), dst_dev = on_device(dst);
    Stager st;
    const size_t o_src = src_dev ? 0 : st.take(in_bytes);
    const size_t o_dst = dst_dev ? 0 : st.take(out_bytes);
    cudaError_t e = sc->ensure(st.used ? st.used : 256);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    char* base = static_cast<char*>(sc->buf);
    const void* dsrc = src_dev ? static_cast<const void*>(src) : base + o_src;
    void* ddst = dst_dev ? dst : base + o_dst;
    if (!src_dev) {
        e = cudaMemcpyAsync(base + o_src, src, in_bytes, cudaMemcpyHostToDevice, sc->stream);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
    }
    e = launch_dequant(type, dsrc, ddst, n, want_f16 != 0, sc->stream);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    if (!dst_dev) {
        e = cudaMemcpyAsync(dst, ddst, out_bytes, cudaMemcpyDeviceToHost, sc->stream);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
    }
    e = cudaStreamSynchronize(sc->stream);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    return ST_OK;
}

int moe_quant_expert(int gate_type, const uint8_t* gate, int64_t gate_bytes,
                     int up_type, const uint8_t* up, int64_t up_bytes,
                     int down_type, const uint8_t* down, int64_t down_bytes,
                     const float* input, int hidden, int intermediate, float* output,
                     int fp16_graph) {
    // argument checks in the reference's order (cpp/moe_quant_dot.cpp:177-188)
    const int types[3] = {gate_type, up_type, down_type};
    const int cols[3] = {hidden, hidden, intermediate};
    const int rows[3] = {intermediate, intermediate, hidden};
    const int64_t sizes[3] = {gate_bytes, up_bytes, down_bytes};
    if (!gate || !up || !down || !input || !output || hidden <= 0 || intermediate <= 0 ||
        hidden > 65536 || intermediate > 65536 || (fp16_graph != 0 && fp16_graph != 1))
        return ST_ARG;
    for (int i = 0; i < 3; ++i) {
        const int bs = block_size(types[i]);
        if (!bs || cols[i] % bs) return ST_TYPE;
        if (sizes[i] != (int64_t)rows[i] * (cols[i] / bs) * block_bytes(types[i])) return ST_BYTES;
    }
    try {
        Scratch* sc = thread_scratch();
        if (!sc) return fail(cudaErrorInvalidDevice, ST_INTERNAL);
        const void* ptrs[4] = {gate, up, down, input};
        const size_t bytes[4] = {(size_t)gate_bytes, (size_t)up_bytes, (size_t)down_bytes,
                                 (size_t)hidden * 4};
        bool dev[4];
        size_t off[4];
        Stager st;
        for (int i = 0; i < 4; ++i) {
            dev[i] = on_device(ptrs[i]) && aligned16(ptrs[i]);
            off[i] = dev[i] ? 0 : st.take(bytes[i]);
        }
        const size_t o_act = st.take((size_t)2 * intermediate * 4);
        const size_t o_y = st.take((size_t)hidden * 4);
        const size_t o_res = st.take(16);
        cudaError_t e = sc->ensure(st.used);
        if (e == cudaSuccess) e = sc->ensure_host((size_t)hidden * 4 + 16);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        char* base = static_cast<char*>(sc->buf);
        const void* dptr[4];
        for (int i = 0; i < 4; ++i) {
            if (dev[i]) {
                dptr[i] = ptrs[i];
            } else {
                e = cudaMemcpyAsync(base + off[i], ptrs[i], bytes[i], cudaMemcpyDefault,
                                    sc->stream);
                if (e != cudaSuccess) return fail(e, ST_INTERNAL);
                dptr[i] = base + off[i];
            }
        }
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
        p.x = static_cast<const float*>(dptr[3]);
        p.gate = qmat(gate_type, dptr[0], intermediate, hidden);
        p.up = qmat(up_type, dptr[1], intermediate, hidden);
        p.down = qmat(down_type, dptr[2], hidden, intermediate);
        p.act = reinterpret_cast<float*>(base + o_act);
        p.y = reinterpret_cast<float*>(base + o_y);
        e = launch_exact(p, sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        // rows up to and including the first non-finite one are written,
        // as the reference's output loop stops there (moe_quant_dot.cpp:207-211)
        int* res_h = reinterpret_cast<int*>(static_cast<char*>(sc->host) + (size_t)hidden * 4);
        if (((uintptr_t)output & 3u) == 0 && on_this_device(output)) {
            int* res_d = reinterpret_cast<int*>(base + o_res);
            k_emit_rows<<<1, 256, 0, sc->stream>>>(p.y, output, hidden, res_d);
            e = cudaGetLastError();
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(res_h, res_d, 8, cudaMemcpyDeviceToHost, sc->stream);
            if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
            if (e != cudaSuccess) return fail(e, ST_INTERNAL);
            return res_h[1] ? ST_NONFINITE : ST_OK;
        }
        float* y = static_cast<float*>(sc->host);
        e = cudaMemcpyAsync(y, p.y, (size_t)hidden * 4, cudaMemcpyDeviceToHost, sc->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        int n_out = hidden, status = ST_OK;
        for (int r = 0; r < hidden; ++r) {
            if (!std::isfinite(y[r])) {
                n_out = r + 1;
                status = ST_NONFINITE;
                break;
            }
        }
        if (on_device(output)) {
            e = cudaMemcpy(output, y, (size_t)n_out * 4, cudaMemcpyHostToDevice);
            if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        } else {
            std::memcpy(output, y, (size_t)n_out * 4);
        }
        return status;
    } catch (...) {
        return ST_INTERNAL;
    }
}

// Argument checks of moe_delta_heads, in the reference's terms
// (cpp/moe_delta.cpp:21-24).
static bool delta_args_ok(const void* const* ptrs, int heads, int dk, int dv) {
    for (int i = 0; i < 7; ++i)
        if (!ptrs[i]) return false;
    return heads >= 1 && heads <= 256 && dk >= 1 && dk <= 1024 && dv >= 1 && dv <= 1024;
}

static constexpr int DELTA_NONFINITE = -2;  // cpp/moe_delta.cpp:66

int moe_delta_heads(float* state, const float* q, const float* k, const float* v,
                    const float* beta, const float* gate, float* output, int heads,
                    int key_dim, int value_dim) {
    const void* all[7] = {state, q, k, v, beta, gate, output};
    if (!delta_args_ok(all, heads, key_dim, value_dim)) return ST_ARG;
    try {
        bool any_device = false;
        for (const void* p : all) any_device = any_device || on_device(p);
        if (!any_device) {   // the reference caller's form: every array on the host
            cudaError_t ce = cudaSuccess;
            const int rc = delta_heads_host(state, q, k, v, beta, gate, output, heads, key_dim,
                                            value_dim, &ce);
            return rc == ST_INTERNAL ? fail(ce, ST_INTERNAL) : rc;
        }
        Scratch* sc = thread_scratch();
        if (!sc) return fail(cudaErrorInvalidDevice, ST_INTERNAL);
        const size_t rows = (size_t)heads * value_dim;
        const size_t row_bytes = (size_t)key_dim * 4;
        // state, q, k, v, beta: used in place when on the device, else staged
        const void* ptrs[5] = {state, q, k, v, beta};
        const size_t bytes[5] = {rows * row_bytes, (size_t)heads * row_bytes,
                                 (size_t)heads * row_bytes, rows * 4, (size_t)heads * 4};
        bool dev[5];
        size_t off[5];
        Stager st;
        for (int i = 0; i < 5; ++i) {
            dev[i] = on_device(ptrs[i]) && ((uintptr_t)ptrs[i] & 3u) == 0;
            off[i] = dev[i] ? 0 : st.take(bytes[i]);
        }
        const size_t o_decay = st.take((size_t)heads * 8);
        const size_t o_out = st.take(rows * 4);
        const size_t o_bad = st.take(8);   // first non-finite row, timeout word
        cudaError_t e = sc->ensure(st.used);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        char* base = static_cast<char*>(sc->buf);
        void* dptr[5];
        for (int i = 0; i < 5; ++i) {
            if (dev[i]) {
                dptr[i] = const_cast<void*>(ptrs[i]);
            } else {
                dptr[i] = base + off[i];
                e = cudaMemcpyAsync(dptr[i], ptrs[i], bytes[i], cudaMemcpyDefault, sc->stream);
                if (e != cudaSuccess) return fail(e, ST_INTERNAL);
            }
        }
        // decay = exp(double(gate)) on the host, with the same libm as the
        // reference's std::exp, so the decayed state has its bits
        std::vector<float> g(heads);
        e = cudaMemcpyAsync(g.data(), gate, (size_t)heads * 4, cudaMemcpyDefault, sc->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        std::vector<double> decay(heads);
        for (int h = 0; h < heads; ++h) decay[h] = std::exp(static_cast<double>(g[h]));
        e = cudaMemcpyAsync(base + o_decay, decay.data(), (size_t)heads * 8,
                            cudaMemcpyHostToDevice, sc->stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(base + o_bad, 0xFF, 4, sc->stream);
        if (e == cudaSuccess) e = cudaMemsetAsync(base + o_bad + 4, 0, 4, sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        DeltaArgs a{};
        a.state = static_cast<float*>(dptr[0]);
        a.q = static_cast<const float*>(dptr[1]);
        a.k = static_cast<const float*>(dptr[2]);
        a.v = static_cast<const float*>(dptr[3]);
        a.beta = static_cast<const float*>(dptr[4]);
        a.gate = nullptr;
        a.decay = reinterpret_cast<const double*>(base + o_decay);
        a.out = reinterpret_cast<float*>(base + o_out);
        a.bad = reinterpret_cast<unsigned*>(base + o_bad);
        a.err = a.bad + 1;
        a.heads = heads;
        a.dk = key_dim;
        a.dv = value_dim;
        e = launch_delta_heads(a, sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        unsigned words[2] = {0, 0};
        e = cudaMemcpyAsync(words, a.bad, 8, cudaMemcpyDeviceToHost, sc->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        if (words[1]) return ST_TIMEOUT;
        const unsigned bad = words[0];
        // the reference stops at the first non-finite output: rows up to and
        // including it hold their new state, later rows keep the old one, and
        // outputs are written for the rows before it (cpp/moe_delta.cpp:64-67)
        const bool ok = bad == 0xFFFFFFFFu;
        const size_t n_state = ok ? rows : (size_t)bad + 1;
        const size_t n_out = ok ? rows : (size_t)bad;
        if (!dev[0]) {
            e = cudaMemcpyAsync(state, a.state, n_state * row_bytes, cudaMemcpyDefault, sc->stream);
            if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        }
        if (n_out) {
            e = cudaMemcpyAsync(output, a.out, n_out * 4, cudaMemcpyDefault, sc->stream);
            if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        }
        e = cudaStreamSynchronize(sc->stream);
        if (e != cudaSuccess) return fail(e, ST_INTERNAL);
        return ok ? ST_OK : DELTA_NONFINITE;
    } catch (...) {
        return ST_INTERNAL;
    }
}

int moe_b200_delta_heads(float* state, const float* q, const float* k, const float* v,
                         const float* beta, const float* gate, float* output, int heads,
                         int key_dim, int value_dim, int32_t* status, void* stream) {
    const void* all[7] = {state, q, k, v, beta, gate, output};
    if (!delta_args_ok(all, heads, key_dim, value_dim)) return ST_ARG;
    for (const void* p : all)
        if ((uintptr_t)p & 3u) return ST_ALIGN;
    if ((uintptr_t)status & 3u) return ST_ALIGN;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (status) {
        cudaError_t e = cudaMemsetAsync(status, 0xFF, 4, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(status + 1, 0, 4, s);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
    }
    DeltaArgs a{};
    a.state = state;
    a.q = q;
    a.k = k;
    a.v = v;
    a.beta = beta;
    a.gate = gate;
    a.decay = nullptr;
    a.out = output;
    a.bad = reinterpret_cast<unsigned*>(status);
    a.err = status ? reinterpret_cast<unsigned*>(status + 1) : nullptr;
    a.heads = heads;
    a.dk = key_dim;
    a.dv = value_dim;
    cudaError_t e = launch_delta_heads(a, s);
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_dequant(int type, const void* src, void* dst, int64_t n, int out_dtype,
                     void* stream) {
    const int bs = block_size(type);
    if (bs == 0 || !src || !dst || n <= 0 || n % bs || (out_dtype != 0 && out_dtype != 1))
        return ST_ARG;
    cudaError_t e = launch_dequant(type, src, dst, n, out_dtype == 1,
                                   static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_decode_kernels(const moe_b200_layer* L, int32_t T, int* kernels) {
    const int st = check_layer(L);
    if (st != ST_OK) return st;
    if (T < 1 || !kernels) return ST_ARG;
    if (fused_supported(L, T, L->flags) || multi_supported(L, T, L->flags)) {
        *kernels = 1;
    } else {
        const bool shared_only = (L->flags & MOE_B200_SHARED_ONLY) != 0;
        *kernels = (shared_only ? 1 : 2) + 2;  // [scores,] top-k/gate, gate/up, down
    }
    return ST_OK;
}

int moe_b200_decode_workspace(const moe_b200_layer* L, int32_t max_tokens, size_t* bytes) {
    const int st = check_layer(L);
    if (st != ST_OK) return st;
    if (max_tokens < 1 || !bytes) return ST_ARG;
    *bytes = decode_ws(L, max_tokens).total;
    return ST_OK;
}

// Staging rows of moe_b200_decode_host after the decode workspace.
struct HostWs {
    size_t x, y, ids, w, total;
};

static HostWs host_ws(const moe_b200_layer* L, int T) {
    Stager s;
    s.used = align_up(decode_ws(L, T).total);
    HostWs h;
    h.x = s.take((size_t)T * L->hidden * 4);
    h.y = s.take((size_t)T * L->hidden * 4);
    h.ids = s.take((size_t)T * L->top_k * 4);
    h.w = s.take((size_t)T * L->top_k * 4);
    h.total = s.used;
    return h;
}

int moe_b200_decode_host_workspace(const moe_b200_layer* L, int32_t max_tokens, size_t* bytes) {
    const int st = check_layer(L);
    if (st != ST_OK) return st;
    if (max_tokens < 1 || !bytes) return ST_ARG;
    *bytes = host_ws(L, max_tokens).total;
    return ST_OK;
}

// This thread's pinned staging rows of moe_b200_decode_host's single-token
// path: the token, the result, the routing and the error word, which the
// device reads and writes through the pinned mapping.
struct HostStage {
    float* x = nullptr;
    float* y = nullptr;
    int32_t* ids = nullptr;
    float* w = nullptr;
    int* err = nullptr;
    int H = 0, K = 0;
};

static cudaError_t host_stage(HostStage& hs, int H, int K) {
    if (hs.x && hs.H >= H && hs.K >= K) return cudaSuccess;
    if (hs.x) cudaFreeHost(hs.x);
    hs = HostStage{};
    const size_t rows = (size_t)H * 4, kb = ((size_t)K * 4 + 15) & ~(size_t)15;
    char* b = nullptr;
    cudaError_t e = cudaMallocHost(reinterpret_cast<void**>(&b), 2 * rows + 2 * kb + 16);
    if (e != cudaSuccess) return e;
    hs.x = reinterpret_cast<float*>(b);
    hs.y = reinterpret_cast<float*>(b + rows);
    hs.ids = reinterpret_cast<int32_t*>(b + 2 * rows);
    hs.w = reinterpret_cast<float*>(b + 2 * rows + kb);
    hs.err = reinterpret_cast<int*>(b + 2 * rows + 2 * kb);
    hs.H = H;
    hs.K = K;
    return cudaSuccess;
}

int moe_b200_decode_host(const moe_b200_layer* L, const float* x, int32_t T, float* y,
                         int32_t* topk_ids, float* topk_weights, void* workspace,
                         size_t workspace_bytes, void* stream) {
    int st = check_layer(L);
    if (st != ST_OK) return st;
    if (T < 1 || !x || !y || !workspace) return ST_ARG;
    if ((uintptr_t)workspace & 255u) return ST_ALIGN;
    const HostWs hw = host_ws(L, T);
    if (workspace_bytes < hw.total) return ST_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* base = static_cast<char*>(workspace);
    float* xd = reinterpret_cast<float*>(base + hw.x);
    float* yd = reinterpret_cast<float*>(base + hw.y);
    int32_t* idd = topk_ids ? reinterpret_cast<int32_t*>(base + hw.ids) : nullptr;
    float* wd = topk_weights ? reinterpret_cast<float*>(base + hw.w) : nullptr;
    const size_t xb = (size_t)T * L->hidden * 4, kb = (size_t)T * L->top_k * 4;
    static thread_local HostStage hs;
    cudaError_t e = host_stage(hs, L->hidden, L->top_k);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    // one token: the token goes through the pinned staging row, one graph
    // launch (a copy-in kernel and the fused kernel, which writes the result,
    // the routing and the error word straight to the pinned rows), one
    // synchronisation, and the result is copied out on the host
    if (T == 1 && fused_supported(L, T, L->flags)) {
        memcpy(hs.x, x, xb);
        // the kernel's last CTA replaces this with the error word once every
        // result row is in host memory (system-scope release): the host
        // polls it instead of waking up from a stream synchronisation, for
        // at most kHostPollSeconds, then synchronises the stream (which also
        // reports a failed launch)
        constexpr int kPending = 0x7fffffff;
        constexpr double kHostPollSeconds = 2.0;
        volatile int* done = hs.err;
        *done = kPending;
        bool launched = false;
        e = launch_decode_fused_host(L, L->flags, hs.x, xd, hs.y, hs.ids, hs.w, hs.err, workspace,
                                     s, &launched);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
        if (launched) {
            const auto t0 = std::chrono::steady_clock::now();
            bool seen = false;
            for (uint32_t i = 0;; ++i) {
                if (*done != kPending) {
                    seen = true;
                    break;
                }
                if ((i & 255u) == 0 &&
                    std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() >
                        kHostPollSeconds)
                    break;
            }
            if (!seen) {
                e = cudaStreamSynchronize(s);
                if (e != cudaSuccess) return fail(e, ST_CUDA);
                if (*done == kPending) return ST_TIMEOUT;
            }
            memcpy(y, hs.y, xb);
            if (topk_ids) memcpy(topk_ids, hs.ids, kb);
            if (topk_weights) memcpy(topk_weights, hs.w, kb);
            return *done;
        }
    }
    int* word_h = hs.err;
    *word_h = 0;
    e = cudaMemcpyAsync(xd, x, xb, cudaMemcpyHostToDevice, s);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    st = moe_b200_decode(L, xd, T, yd, idd, wd, workspace, hw.x, stream);
    if (st != ST_OK) {
        cudaStreamSynchronize(s);
        return st;
    }
    e = cudaMemcpyAsync(y, yd, xb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && idd) e = cudaMemcpyAsync(topk_ids, idd, kb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess && wd) e = cudaMemcpyAsync(topk_weights, wd, kb, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaMemcpyAsync(word_h, base + 32, sizeof(int), cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    const int word = *word_h;
    if (word != 0) {
        e = cudaMemsetAsync(base + 32, 0, sizeof(int), s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        return e == cudaSuccess ? word : fail(e, ST_CUDA);
    }
    return ST_OK;
}

int moe_b200_decode(const moe_b200_layer* L, const float* x, int32_t T, float* y,
                    int32_t* topk_ids, float* topk_weights, void* workspace,
                    size_t workspace_bytes, void* stream) {
    int st = check_layer(L);
    if (st != ST_OK) return st;
    if (T < 1 || !x || !y || !workspace) return ST_ARG;
    if (!aligned16(x) || !aligned16(y) || ((uintptr_t)workspace & 255u)) return ST_ALIGN;
    const DecodeWs ws = decode_ws(L, T);
    if (workspace_bytes < ws.total) return ST_WORKSPACE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    char* base = static_cast<char*>(workspace);
    const bool shared_only = (L->flags & MOE_B200_SHARED_ONLY) != 0;
    const bool with_shared = L->shared_intermediate > 0 && !(L->flags & MOE_B200_NO_SHARED);
    if (shared_only && !with_shared) return ST_ARG;

    if (fused_supported(L, T, L->flags)) {
        bool launched = false;
        cudaError_t fe = launch_decode_fused(L, L->flags, x, y, topk_ids, topk_weights, workspace, s,
                                             &launched);
        if (fe != cudaSuccess) return fail(fe, ST_CUDA);
        if (launched) return ST_OK;
    } else if (multi_supported(L, T, L->flags)) {
        bool launched = false;
        cudaError_t fe = launch_decode_multi(L, L->flags, x, T, 0, T, y, topk_ids, topk_weights,
                                             workspace, s, &launched);
        if (fe != cudaSuccess) return fail(fe, ST_CUDA);
        if (launched) return ST_OK;
    }

    RoutePlan r{};
    r.T = T;
    r.E = L->n_experts;
    r.K = shared_only ? 0 : L->top_k;
    r.H = L->hidden;
    r.x = x;
    r.router = L->router;
    r.bias = L->router_bias;
    r.gate_inp = with_shared ? L->shared_gate_inp : nullptr;
    r.scores = reinterpret_cast<float*>(base + ws.scores);
    r.ids = reinterpret_cast<int32_t*>(base + ws.ids);
    r.w = reinterpret_cast<float*>(base + ws.w);
    r.sg = reinterpret_cast<float*>(base + ws.sg);
    cudaError_t e = launch_route(r, s);
    if (e != cudaSuccess) return fail(e, ST_CUDA);

    ExactPlan p{};
    p.T = T;
    p.K = L->top_k;
    p.H = L->hidden;
    p.I = L->intermediate;
    p.Is = with_shared ? L->shared_intermediate : 0;
    p.Imax = L->shared_intermediate > L->intermediate ? L->shared_intermediate : L->intermediate;
    p.round16 = (L->flags & MOE_B200_FP16_GRAPH) ? 1 : 0;
    p.expert_begin = L->expert_begin;
    p.expert_count = shared_only ? 0 : L->expert_count;
    p.x = x;
    p.ids = r.ids;
    p.w = r.w;
    p.sg = with_shared ? r.sg : nullptr;
    p.gate = qmat(L->gate_type, L->gate, L->intermediate, L->hidden);
    p.up = qmat(L->up_type, L->up, L->intermediate, L->hidden);
    p.down = qmat(L->down_type, L->down, L->hidden, L->intermediate);
    if (with_shared) {
        p.sgate = qmat(L->shared_gate_type, L->shared_gate, L->shared_intermediate, L->hidden);
        p.sup = qmat(L->shared_up_type, L->shared_up, L->shared_intermediate, L->hidden);
        p.sdown = qmat(L->shared_down_type, L->shared_down, L->hidden, L->shared_intermediate);
    }
    p.act = reinterpret_cast<float*>(base + ws.act);
    p.y = y;
    e = launch_exact(p, s);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    if (topk_ids && !shared_only) {
        e = cudaMemcpyAsync(topk_ids, r.ids, (size_t)T * L->top_k * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
    }
    if (topk_weights && !shared_only) {
        e = cudaMemcpyAsync(topk_weights, r.w, (size_t)T * L->top_k * 4, cudaMemcpyDeviceToDevice, s);
        if (e != cudaSuccess) return fail(e, ST_CUDA);
    }
    return ST_OK;
}

int moe_b200_block_prepare(const float* x, float* h, float* n, int32_t T, int32_t H, float eps,
                           void* stream) {
    if (!x || !h || !n || T < 1 || H < 1 || !(eps >= 0.f)) return ST_ARG;
    cudaError_t e = launch_block_prepare(x, h, n, T, H, eps, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_block_finish(const float* h, const float* m, float* y, int32_t T, int32_t H,
                          void* stream) {
    if (!h || !m || !y || T < 1 || H < 1) return ST_ARG;
    cudaError_t e = launch_block_finish(h, m, y, T, H, static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? ST_OK : fail(e, ST_CUDA);
}

int moe_b200_decode_steps(const moe_b200_layer* L0, const moe_b200_layer* layers,
                          const moe_b200_step* steps, int32_t n_steps, float eps, void* workspace,
                          size_t workspace_bytes, void* stream) {
    int st = check_layer(L0);
    if (st != ST_OK) return st;
    if (!layers || !steps || n_steps < 1 || !workspace || !(eps >= 0.f)) return ST_ARG;
    if (((uintptr_t)workspace & 255u) || ((uintptr_t)steps & 15u) || ((uintptr_t)layers & 15u))
        return ST_ALIGN;
    if (!fused_supported(L0, 1, L0->flags)) return ST_TYPE;
    if (workspace_bytes < decode_ws(L0, 1).total) return ST_WORKSPACE;
    bool launched = false;
    cudaError_t e = launch_decode_steps(L0, layers, steps, n_steps, eps, workspace,
                                        static_cast<cudaStream_t>(stream), &launched);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    return launched ? ST_OK : ST_TYPE;
}

int moe_b200_decode_ep(const moe_b200_layer* L, const float* x, int32_t T, int32_t shared_begin,
                       int32_t shared_count, float* y, int32_t* topk_ids, float* topk_weights,
                       void* workspace, size_t workspace_bytes, void* stream) {
    int st = check_layer(L);
    if (st != ST_OK) return st;
    if (T < 1 || !x || !y || !workspace) return ST_ARG;
    if (L->flags & (MOE_B200_SHARED_ONLY | MOE_B200_NO_SHARED)) return ST_ARG;
    if (shared_begin < 0 || shared_count < 0 || shared_begin + shared_count > T) return ST_ARG;
    if (shared_count > 0 && L->shared_intermediate <= 0) return ST_ARG;
    if (!aligned16(x) || !aligned16(y) || ((uintptr_t)workspace & 255u)) return ST_ALIGN;
    if (!multi_supported(L, T, L->flags)) return ST_TYPE;
    if (workspace_bytes < decode_ws(L, T).total) return ST_WORKSPACE;
    bool launched = false;
    cudaError_t e = launch_decode_multi(L, L->flags, x, T, shared_begin, shared_begin + shared_count,
                                        y, topk_ids, topk_weights, workspace,
                                        static_cast<cudaStream_t>(stream), &launched);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    return launched ? ST_OK : ST_TYPE;
}

int moe_b200_ep_create(int32_t world, int32_t rank, int32_t tokens_per_rank, int32_t hidden,
                       moe_b200_ep** ctx, void* blob) {
    if (!ctx || !blob) return ST_ARG;
    cudaError_t ce = cudaSuccess;
    const int st = ep_create(world, rank, tokens_per_rank, hidden, ctx, blob, &ce);
    return st == ST_CUDA ? fail(ce, ST_CUDA) : st;
}

int moe_b200_ep_connect(moe_b200_ep* ctx, const void* blobs) {
    cudaError_t ce = cudaSuccess;
    const int st = ep_connect(ctx, blobs, &ce);
    return st == ST_CUDA ? fail(ce, ST_CUDA) : st;
}

int moe_b200_ep_destroy(moe_b200_ep* ctx) {
    if (!ctx) return ST_ARG;
    ep_destroy(ctx);
    return ST_OK;
}

int moe_b200_decode_ep_p2p(const moe_b200_layer* L, moe_b200_ep* ctx, const float* x, float* y,
                           int32_t* topk_ids, float* topk_weights, void* workspace,
                           size_t workspace_bytes, void* stream) {
    int st = check_layer(L);
    if (st != ST_OK) return st;
    if (!ctx || !x || !y || !workspace) return ST_ARG;
    if (!ctx->connected || L->hidden != ctx->H) return ST_ARG;
    if (L->flags & (MOE_B200_SHARED_ONLY | MOE_B200_NO_SHARED)) return ST_ARG;
    if (!aligned16(x) || !aligned16(y) || ((uintptr_t)workspace & 255u)) return ST_ALIGN;
    const int T = ctx->world * ctx->tq;
    if (!multi_supported(L, T, L->flags)) return ST_TYPE;
    if (workspace_bytes < decode_ws(L, T).total) return ST_WORKSPACE;
    bool launched = false;
    cudaError_t e = launch_decode_multi(L, L->flags, x, T, 0, 0, y, topk_ids, topk_weights,
                                        workspace, static_cast<cudaStream_t>(stream), &launched,
                                        ctx);
    if (e != cudaSuccess) return fail(e, ST_CUDA);
    return launched ? ST_OK : ST_TYPE;
}

int moe_b200_prefill_supported(const moe_b200_layer* L) {
    if (check_layer(L) != ST_OK) return 0;
    return prefill_supported(L, L->flags) ? 1 : 0;
}

int moe_b200_prefill_workspace(const moe_b200_layer* L, int32_t max_tokens, size_t* bytes) {
    const int st = check_layer(L);
    if (st != ST_OK) return st;
    if (max_tokens < 1 || !bytes) return ST_ARG;
    *bytes = prefill_workspace_bytes(L, max_tokens);
    return ST_OK;
}

int moe_b200_prefill(const moe_b200_layer* L, const void* x, int32_t x_dtype, int32_t T,
                     float* y, int32_t* topk_ids, float* topk_weights, void* workspace,
                     size_t workspace_bytes, void* stream) {
    int st = check_layer(L);
    if (st != ST_OK) return st;
    if (T < 1 || !x || !y || !workspace || (x_dtype != 0 && x_dtype != 1)) return ST_ARG;
    if (!aligned16(x) || !aligned16(y) || ((uintptr_t)workspace & 255u)) return ST_ALIGN;
    const bool shared_only = (L->flags & MOE_B200_SHARED_ONLY) != 0;
    const bool with_shared = L->shared_intermediate > 0 && !(L->flags & MOE_B200_NO_SHARED);
    if (shared_only && !with_shared) return ST_ARG;
    if (!prefill_supported(L, L->flags)) return ST_TYPE;
    if (workspace_bytes < prefill_workspace_bytes(L, T)) return ST_WORKSPACE;
    cudaError_t ce = cudaSuccess;
    st = prefill_run(L, x, x_dtype, T, y, topk_ids, topk_weights, workspace, workspace_bytes,
                     static_cast<cudaStream_t>(stream), &ce);
    if (st == ST_CUDA) return fail(ce, ST_CUDA);
    return st;
}

int moe_b200_prefill_kernels(const moe_b200_layer* L, int tokens, int* kernels) {
    const int st = check_layer(L);
    if (st != ST_OK) return st;
    if (!kernels || tokens <= 0) return ST_ARG;
    *kernels = prefill_kernels(L, tokens);
    return ST_OK;
}

}  // extern "C"
