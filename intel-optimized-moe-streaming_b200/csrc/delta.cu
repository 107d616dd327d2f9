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

}  // namespace

cudaError_t launch_delta_heads(const DeltaArgs& a, cudaStream_t s) {
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
