// sm100.cuh -- Blackwell primitives used by the fused kernels: mbarriers,
// TMA bulk copies (cp.async.bulk, no multicast), acquire/release flags with
// bounded waits.
#pragma once

#include "common.cuh"

namespace moeb200 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait on an mbarrier phase.  Returns false after `limit` polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    return false;
}

// One-dimensional TMA copy global -> shared, completion counted on `bar`.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// One-dimensional TMA copy shared -> global in the thread's bulk group.
// dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
                 ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void bulk_commit() {
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Wait until every bulk group of this thread has completed.
__device__ __forceinline__ void bulk_wait_all() {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Orders this thread's earlier generic-proxy accesses of shared memory
// before later async-proxy (TMA) accesses: before a bulk copy out of shared
// memory this thread wrote, or (after a barrier) into shared memory that
// other threads have read.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_add(uint32_t* p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin (one thread) until *flag >= target, at most `limit` polls.
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t target, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if (ld_acquire(flag) >= target) return true;
    }
    return false;
}

// System-scope flag operations for flags in memory that another GPU writes
// or reads over NVLink (peer mappings of device memory).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Spin (one thread) until *flag >= target (a flag a peer GPU sets), at most
// `limit` polls.
__device__ __forceinline__ bool wait_flag_sys(const uint32_t* flag, uint32_t target, uint32_t limit) {
    for (uint32_t i = 0; i < limit; ++i) {
        if ((int32_t)(ld_acquire_sys(flag) - target) >= 0) return true;
    }
    return false;
}

// One exchange word for memory another GPU reads: a 32-bit payload in the
// low half and the step number in the high half, written with one 64-bit
// store (single-copy atomic), so a reader that sees the step number also
// sees the payload -- no fence or separate flag.
__device__ __forceinline__ void st_word_sys(uint64_t* p, float v, uint32_t seq) {
    const uint64_t w = ((uint64_t)seq << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word_sys(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Two consecutive system-scope exchange words (p 16-byte aligned) in one
// load; each 64-bit element is read whole.
__device__ __forceinline__ ulonglong2 ld_word2_sys(const uint64_t* p) {
    ulonglong2 w;
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}

// Payload of the exchange word at p once it carries step `seq`; at most
// `limit` polls while *ok (cleared when the limit is hit, so a thread that
// gave up once stops waiting).
__device__ __forceinline__ float wait_word_sys(const uint64_t* p, uint32_t seq, uint32_t limit,
                                               bool& ok) {
    uint64_t w = ld_word_sys(p);
    if (ok && (uint32_t)(w >> 32) != seq) {
        uint32_t i = 0;
        for (; i < limit; ++i) {
            w = ld_word_sys(p);
            if ((uint32_t)(w >> 32) == seq) break;
        }
        if (i == limit) ok = false;
    }
    return __uint_as_float((uint32_t)w);
}

// The same exchange word between the CTAs of one GPU (gpu scope): the
// payload and the step tag arrive together, so a CTA that polls the words it
// needs waits for exactly those values, with no release fence on the writer
// side and no counter round trip before the data read.
__device__ __forceinline__ void st_word_gpu(uint64_t* p, float v, uint32_t tag) {
    const uint64_t w = ((uint64_t)tag << 32) | (uint64_t)__float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}

__device__ __forceinline__ uint64_t ld_word_gpu(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}

// Two consecutive exchange words (p 16-byte aligned) in one load; each
// 64-bit element is read whole.
__device__ __forceinline__ ulonglong2 ld_word2_gpu(const uint64_t* p) {
    ulonglong2 w;
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(w.x), "=l"(w.y) : "l"(p) : "memory");
    return w;
}

// Payload of the gpu-scope exchange word at p once it carries `tag` (at most
// `limit` polls while ok; ok is cleared when the limit is hit).
__device__ __forceinline__ float wait_word_gpu(const uint64_t* p, uint32_t tag, uint32_t limit,
                                               bool& ok) {
    uint64_t w = ld_word_gpu(p);
    if (ok && (uint32_t)(w >> 32) != tag) {
        uint32_t i = 0;
        for (; i < limit; ++i) {
            w = ld_word_gpu(p);
            if ((uint32_t)(w >> 32) == tag) break;
        }
        if (i == limit) ok = false;
    }
    return __uint_as_float((uint32_t)w);
}

// Programmatic dependent launch, at the top of a kernel: let the stream's
// next kernel begin launching, then wait until the previous kernel has
// completed and its writes are visible (both no-ops when the launch was not
// programmatic).  Every block of the kernel is resident or done before the
// next one can launch, so its waiting blocks never hold back this kernel.
__device__ __forceinline__ void pdl_enter() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

}  // namespace moeb200
