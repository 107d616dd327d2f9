// One gated delta-rule (DeltaNet) decode step over every head's fp32 state,
// the reference's moe_delta_heads (cpp/moe_delta.cpp:18-69) on sm_100a.
//
// State layout in HBM: [heads][value_dim][key_dim] fp32, one key_dim row per
// (head, value row) -- the reference's layout, so the state needs no
// conversion at the boundary.  Per head h, decay = exp(double(gate[h])); per
// row r:
//   row[j]  <- float(double(row[j]) * decay)
//   kv       = sum_j row[j] * k[h][j]
//   delta    = beta[h] * (v[h][r] - kv)
//   row[j]  <- row[j] + delta * k[h][j]                  (stored)
//   out[h][r] = sum_j row[j] * q[h][j]
//
// The reference sums kv and out in eight lanes (lane = j % 8, one multiply
// then one add per term, lanes summed 0..7 into zero) and then the tail
// j >= key_dim - key_dim % 8 in order.  To give the same bits, eight threads
// own one row, thread l owning lane l: each runs its lane's sum in the
// reference's order, the lane sums are gathered by shuffles and added 0..7 in
// every thread, and the tail is added in every thread.  Every operation is
// an explicitly rounded intrinsic (no contraction).  The decayed row stays
// in registers between the two passes (up to the 1024-value limit), so each
// state byte is read once and written once: the step is HBM bound at
// 8 * heads * value_dim * key_dim bytes.
//
// A non-finite output records the smallest flat row index h * value_dim + r
// in a device word (atomicMin); the host entry point uses it to reproduce
// the reference's early stop exactly.
#include "common.cuh"
#include "launch.h"
#include "sm100.cuh"

namespace moeb200 {

namespace {

constexpr int kDeltaThreads = 128;             // 16 rows per CTA, 4 per warp
constexpr int kDeltaRowsPerWarp = 4;

__device__ __forceinline__ float decay_value(float x, double decay) {
    return __double2float_rn(__dmul_rn(static_cast<double>(x), decay));
}

// sum8 of the reference: lanes 0..7 of this 8-thread group added into zero.
__device__ __forceinline__ float lane_sum8(float acc) {
    float s = 0.0f;
#pragma unroll
    for (int l = 0; l < 8; ++l) s = __fadd_rn(s, __shfl_sync(0xffffffffu, acc, l, 8));
    return s;
}

// Each thread holds its lane of up to NC whole chunks of eight in registers
// (NC * 8 >= key_dim - key_dim % 8), so every state byte is read once and
// written once.  All loads of a row (state, k, q, tail, v, beta, gate) are
// issued before the first use; with NC <= 32 k and q stay in registers too,
// wider rows re-read them from L1 (one head's k and q serve all its rows).
template <int NC>
__global__ void __launch_bounds__(kDeltaThreads)
k_delta_heads(DeltaArgs a) {
    constexpr bool kRegKQ = NC <= 32;
    const int lane = threadIdx.x & 7;
    const int sub = (threadIdx.x >> 3) & (kDeltaRowsPerWarp - 1);
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int nwarps = (gridDim.x * blockDim.x) >> 5;
    const int rows = a.heads * a.dv;
    const int dk = a.dk;
    const int whole = dk & ~7;
    const int nc = whole >> 3;
    const int tail = dk - whole;

    // the loop bound is uniform over the warp, so every shuffle has all 32
    // threads; a group past the last row computes on zeros and stores nothing
    for (int base = warp * kDeltaRowsPerWarp; base < rows; base += nwarps * kDeltaRowsPerWarp) {
        const int row = base + sub;
        const bool valid = row < rows;
        const int h = valid ? row / a.dv : 0;
        float* srow = a.state + static_cast<int64_t>(valid ? row : 0) * dk;
        const float* kh = a.k + static_cast<int64_t>(h) * dk;
        const float* qh = a.q + static_cast<int64_t>(h) * dk;

        float x[NC];
        float kr[kRegKQ ? NC : 1];
        float qr[kRegKQ ? NC : 1];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            x[c] = 0.0f;
            if (c < nc && valid) x[c] = __ldcs(srow + 8 * c + lane);
        }
        if constexpr (kRegKQ) {
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                kr[c] = 0.0f;
                qr[c] = 0.0f;
                if (c < nc && valid) {
                    kr[c] = __ldg(kh + 8 * c + lane);
                    qr[c] = __ldg(qh + 8 * c + lane);
                }
            }
        }
        float xt[7], kt[7], qt[7];
#pragma unroll
        for (int t = 0; t < 7; ++t) {
            xt[t] = kt[t] = qt[t] = 0.0f;
            if (t < tail && valid) {
                xt[t] = srow[whole + t];
                kt[t] = __ldg(kh + whole + t);
                qt[t] = __ldg(qh + whole + t);
            }
        }
        const float vr = valid ? __ldg(a.v + row) : 0.0f;
        const float br = valid ? __ldg(a.beta + h) : 0.0f;
        const double decay = a.decay ? a.decay[h] : exp(static_cast<double>(__ldg(a.gate + h)));

        // pass 1: decay, kv lane sum
        float acc = 0.0f;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            if (c < nc) {
                const float kc = kRegKQ ? kr[c] : (valid ? __ldg(kh + 8 * c + lane) : 0.0f);
                x[c] = decay_value(x[c], decay);
                acc = __fadd_rn(acc, __fmul_rn(x[c], kc));
            }
        }
        float kv = lane_sum8(acc);
#pragma unroll
        for (int t = 0; t < 7; ++t) {
            if (t < tail) {
                xt[t] = decay_value(xt[t], decay);
                kv = __fadd_rn(kv, __fmul_rn(xt[t], kt[t]));
            }
        }
        const float delta = __fmul_rn(br, __fsub_rn(vr, kv));

        // pass 2: update, store, output lane sum
        float acc2 = 0.0f;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            if (c < nc && valid) {
                const float kc = kRegKQ ? kr[c] : __ldg(kh + 8 * c + lane);
                const float qc = kRegKQ ? qr[c] : __ldg(qh + 8 * c + lane);
                const float u = __fadd_rn(x[c], __fmul_rn(delta, kc));
                __stcs(srow + 8 * c + lane, u);
                acc2 = __fadd_rn(acc2, __fmul_rn(u, qc));
            }
        }
        float result = lane_sum8(acc2);
#pragma unroll
        for (int t = 0; t < 7; ++t) {
            if (t < tail && valid) {
                const float u = __fadd_rn(xt[t], __fmul_rn(delta, kt[t]));
                if (lane == t) srow[whole + t] = u;
                result = __fadd_rn(result, __fmul_rn(u, qt[t]));
            }
        }
        if (valid && lane == 0) {
            a.out[row] = result;
            if (!isfinite(result) && a.bad) atomicMin(a.bad, static_cast<unsigned>(row));
        }
    }
}

template <int NC>
cudaError_t launch_nc(const DeltaArgs& a, cudaStream_t s) {
    static int per_sm[64] = {0};   // resident CTAs per SM, per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!per_sm[dev]) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k_delta_heads<NC>, kDeltaThreads, 0) !=
                cudaSuccess || n < 1)
            n = 1;
        per_sm[dev] = n;
    }
    const int rows = a.heads * a.dv;
    const int rows_per_cta = kDeltaThreads / 8;
    int grid = (rows + rows_per_cta - 1) / rows_per_cta;
    const int cap = sm_count() * per_sm[dev];   // one wave; the loop strides over the rest
    if (grid > cap) grid = cap;
    k_delta_heads<NC><<<grid, kDeltaThreads, 0, s>>>(a);
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// Streaming variant for states larger than the GPU can hold in flight in
// registers: one persistent CTA per SM walks tiles of ROWS (32, or 16 when
// a wide row leaves room for fewer than three 32-row stages) consecutive
// rows, eight threads per row.
// A tile's rows, and the k and q rows of the heads it touches, arrive in a
// shared-memory stage by TMA bulk copies (one per row, completion counted on
// the stage's mbarrier); the warps compute from shared memory (row stride
// P = key_dim padded to 8 mod 32 floats, so the four rows a warp reads fall
// in distinct banks), keep the decayed row there between the two passes
// (one double multiply per value), write the updated rows back in place,
// and one thread bulk-stores them to HBM.  S stages keep S - 1 tiles of loads in
// flight behind the tile being computed; a stage is refilled once the bulk
// store of its previous tile has finished reading it.  Needs key_dim % 4 == 0
// and 16-byte aligned state, k and q (TMA bulk copy alignment).

constexpr uint32_t kDeltaWaitPolls = 1u << 21;
constexpr int kStreamSmemHead = 256;        // mbarriers and the abort flag
constexpr size_t kStreamSmemMax = 232448;   // 227 KiB dynamic shared memory

struct StreamShape {
    int rows = 0, P = 0, NH = 0, S = 0;
    size_t stage_floats = 0, smem = 0;
};

StreamShape stream_shape(int dk, int dv, int tile_rows) {
    StreamShape sh;
    sh.rows = tile_rows;
    sh.P = dk + ((8 - dk % 32) + 32) % 32;
    const int nh = (tile_rows - 1) / dv + 2;   // heads tile_rows consecutive rows can touch
    sh.NH = nh < tile_rows ? nh : tile_rows;
    sh.stage_floats = (size_t)(tile_rows + 2 * sh.NH) * sh.P;
    const size_t stage_bytes = sh.stage_floats * 4;
    size_t S = (kStreamSmemMax - kStreamSmemHead) / stage_bytes;
    if (S > 8) S = 8;
    sh.S = (int)S;
    sh.smem = kStreamSmemHead + S * stage_bytes;
    return sh;
}

template <int ROWS>
__global__ void __launch_bounds__(ROWS * 8, 1)
k_delta_stream(DeltaArgs a, int P, int NH, int S, int tiles) {
    extern __shared__ __align__(128) unsigned char smem_raw[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw);   // S <= 8 barriers
    volatile int* abort_flag = reinterpret_cast<volatile int*>(smem_raw + 128);
    float* stages = reinterpret_cast<float*>(smem_raw + kStreamSmemHead);
    const size_t stage_floats = (size_t)(ROWS + 2 * NH) * P;

    const int tid = threadIdx.x;
    const int lane = tid & 7;
    const int rsub = tid >> 3;   // row of the tile; warp w holds rows 4w..4w+3
    const int rows = a.heads * a.dv;
    const int dk = a.dk, dv = a.dv;
    const int whole = dk & ~7;
    const int nc = whole >> 3;
    const int tail = dk - whole;
    const uint32_t rb = (uint32_t)dk * 4u;

    if (tid == 0) {
        for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
        mbar_fence_init();
        *abort_flag = 0;
    }
    __syncthreads();

    // tile of this CTA's i-th iteration; issued by thread 0 only
    auto issue = [&](int i) {
        const int t = blockIdx.x + i * gridDim.x;
        if (t >= tiles) return false;
        float* st = stages + (size_t)(i % S) * stage_floats;
        const int r0 = t * ROWS;
        const int n = rows - r0 < ROWS ? rows - r0 : ROWS;
        const int h0 = r0 / dv;
        const int nh = (r0 + n - 1) / dv - h0 + 1;
        uint64_t* bar = &full[i % S];
        mbar_arrive_expect_tx(bar, (uint32_t)(n + 2 * nh) * rb);
        for (int rr = 0; rr < n; ++rr)
            bulk_g2s(st + (size_t)rr * P, a.state + (size_t)(r0 + rr) * dk, rb, bar);
        for (int hh = 0; hh < nh; ++hh) {
            bulk_g2s(st + (size_t)(ROWS + 2 * hh) * P, a.k + (size_t)(h0 + hh) * dk, rb, bar);
            bulk_g2s(st + (size_t)(ROWS + 2 * hh + 1) * P, a.q + (size_t)(h0 + hh) * dk, rb,
                     bar);
        }
        return true;
    };

    int issued = 0;   // thread 0: iterations whose loads are in flight or consumed
    if (tid == 0)
        while (issued < S && issue(issued)) ++issued;

    int i = 0;
    for (;; ++i) {
        const int t = blockIdx.x + i * gridDim.x;
        if (t >= tiles) break;
        const int s = i % S;
        if (tid == 0 && !mbar_wait(&full[s], (uint32_t)(i / S) & 1u, kDeltaWaitPolls)) *abort_flag = 1;
        __syncthreads();
        if (*abort_flag) break;

        float* st = stages + (size_t)s * stage_floats;
        const int r0 = t * ROWS;
        const int n = rows - r0 < ROWS ? rows - r0 : ROWS;
        const bool valid = rsub < n;
        const int row = r0 + (valid ? rsub : 0);
        const int h = row / dv;
        float* xs = st + (size_t)rsub * P;
        const float* ks = st + (size_t)(ROWS + 2 * (h - r0 / dv)) * P;
        const float* qs = ks + P;
        const double decay = a.decay ? a.decay[h] : exp(static_cast<double>(__ldg(a.gate + h)));
        const float vr = __ldg(a.v + row);
        const float br = __ldg(a.beta + h);

        // pass 1 (rows past the tile's end compute on stale shared memory and
        // store nothing; they keep the warp's shuffles complete)
        float acc = 0.0f;
        for (int c = 0; c < nc; ++c) {
            const int j = 8 * c + lane;
            const float d = decay_value(xs[j], decay);
            xs[j] = d;   // this thread's own value: no other thread reads it
            acc = __fadd_rn(acc, __fmul_rn(d, ks[j]));
        }
        float kv = lane_sum8(acc);
        float xt[7];
#pragma unroll
        for (int u = 0; u < 7; ++u) {
            xt[u] = 0.0f;
            if (u < tail) {
                xt[u] = decay_value(xs[whole + u], decay);
                kv = __fadd_rn(kv, __fmul_rn(xt[u], ks[whole + u]));
            }
        }
        const float delta = __fmul_rn(br, __fsub_rn(vr, kv));

        // pass 2 (the tail's decayed values stay in registers: every lane of
        // the row reads the tail, so it is not overwritten before the shuffles)
        float acc2 = 0.0f;
        for (int c = 0; c < nc; ++c) {
            const int j = 8 * c + lane;
            const float u = __fadd_rn(xs[j], __fmul_rn(delta, ks[j]));
            xs[j] = u;
            acc2 = __fadd_rn(acc2, __fmul_rn(u, qs[j]));
        }
        float result = lane_sum8(acc2);
#pragma unroll
        for (int u = 0; u < 7; ++u) {
            if (u < tail) {
                const float nu = __fadd_rn(xt[u], __fmul_rn(delta, ks[whole + u]));
                if (lane == u) xs[whole + u] = nu;
                result = __fadd_rn(result, __fmul_rn(nu, qs[whole + u]));
            }
        }
        if (valid && lane == 0) {
            a.out[row] = result;
            if (!isfinite(result) && a.bad) atomicMin(a.bad, static_cast<unsigned>(row));
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            for (int rr = 0; rr < n; ++rr)
                bulk_s2g(a.state + (size_t)(r0 + rr) * dk, st + (size_t)rr * P, rb);
            bulk_commit();
            if (i >= 1 && issued == i - 1 + S) {
                bulk_wait_read<1>();   // the previous tile's stores have read their stage
                if (issue(issued)) ++issued;
            }
        }
    }
    if (tid == 0) {
        if (*abort_flag) {
            if (a.err) atomicOr(a.err, 1u);
            // loads still in flight land before the CTA's shared memory goes
            for (int j = i; j < issued; ++j) mbar_wait(&full[j % S], (uint32_t)(j / S) & 1u, kDeltaWaitPolls);
        }
        bulk_wait_all();
    }
}

template <int ROWS>
cudaError_t launch_stream(const DeltaArgs& a, const StreamShape& sh, cudaStream_t s) {
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(k_delta_stream<ROWS>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)kStreamSmemMax);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
    }
    const int rows = a.heads * a.dv;
    const int tiles = (rows + ROWS - 1) / ROWS;
    int grid = sm_count();
    if (grid > tiles) grid = tiles;
    k_delta_stream<ROWS><<<grid, ROWS * 8, sh.smem, s>>>(a, sh.P, sh.NH, sh.S, tiles);
    return cudaGetLastError();
}

}  // namespace

// Rows from which the streaming variant is used: four tiles per SM.
constexpr int kStreamMinRowsPerSm = 64;

cudaError_t launch_delta_heads(const DeltaArgs& a, cudaStream_t s) {
    const int rows = a.heads * a.dv;
    const bool aligned = ((uintptr_t)a.state | (uintptr_t)a.k | (uintptr_t)a.q) % 16 == 0;
    if (a.dk % 4 == 0 && aligned && rows >= kStreamMinRowsPerSm * sm_count()) {
        const StreamShape wide = stream_shape(a.dk, a.dv, 32);
        if (wide.S >= 3) return launch_stream<32>(a, wide, s);
        const StreamShape sh = stream_shape(a.dk, a.dv, 16);
        if (sh.S >= 2) return launch_stream<16>(a, sh, s);
    }
    const int nc = a.dk >> 3;
    if (nc <= 1) return launch_nc<1>(a, s);
    if (nc <= 2) return launch_nc<2>(a, s);
    if (nc <= 4) return launch_nc<4>(a, s);
    if (nc <= 8) return launch_nc<8>(a, s);
    if (nc <= 16) return launch_nc<16>(a, s);
    if (nc <= 32) return launch_nc<32>(a, s);
    if (nc <= 64) return launch_nc<64>(a, s);
    return launch_nc<128>(a, s);
}

}  // namespace moeb200
