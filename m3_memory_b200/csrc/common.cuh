// common.cuh -- shared device helpers for the m3gpu kernels (sm_100a).
//
// Everything that waits on the GPU waits with an iteration limit: a wait that
// runs out records an error code in the launch's error word and returns, so a
// broken pipeline ends the kernel with an error status the host reads instead
// of hanging the device.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace m3g {

enum MetricKind : int { kL2 = 0, kIP = 1, kCosine = 2 };

// Error codes a kernel can leave in its error word (0 = none).
enum KernelError : int {
    kErrNone = 0,
    kErrWaitTimeout = 1,   // an mbarrier wait ran past its iteration limit
    kErrBadItem = 2,       // a work item failed its bounds check
    kErrCapacity = 3,      // a fixed-size buffer would have overflowed
};

// Every mbarrier wait gives up after kWaitLimitNs of wall time (%globaltimer).
constexpr uint64_t kWaitLimitNs = 1000000000ull;  // 1 s
// Iteration cap of the waits that must not depend on the timer (drains).
constexpr uint32_t kWaitSpinLimit = 1u << 22;

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------- mbarrier ----------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\t"
        "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
        : "memory");
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

// try_wait that lets the hardware suspend the warp for up to `hint_ns` while
// the phase is incomplete (no issue slots burnt spinning).
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity,
                                                   uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false
// (and records kErrWaitTimeout) when kWaitLimitNs pass, or as soon as another
// thread of the launch has recorded an error.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err,
                                              uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 20000u)) return true;
        if (*(volatile int*)err != 0) return false;
        if (global_ns() - t0 > limit_ns) break;
    }
    atomicCAS(err, 0, (int)kErrWaitTimeout);
    return false;
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
    return mbar_wait_for(bar, parity, err, kWaitLimitNs);
}

// ---------------- bulk / tensor copies (TMA), no multicast ----------------

// 1-D bulk copy global -> shared, completion counted on `bar` (bytes % 16 == 0,
// both addresses 16-byte aligned).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor load (box described by the tensor map) into shared memory.
// x is the innermost coordinate in elements and must keep x*elem_size a
// multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// The same with the destination given as a shared-memory address.
__device__ __forceinline__ void tma_load_2d_u32(uint32_t dst, const CUtensorMap* map, int x, int y,
                                                uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Named barrier over `nthreads` threads (a multiple of 32) with id `id` (1..15).
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over its participants: every thread
// gets the same answer, so a "stop" decision taken here is uniform.
__device__ __forceinline__ bool named_bar_sync_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// ---------------- ordering keys ----------------

// Monotone map float -> uint32 (ascending floats give ascending keys; -0 and +0
// share a key, as they compare equal; NaN sorts after +inf).
__device__ __forceinline__ uint32_t float_key(float f) {
    uint32_t u = __float_as_uint(f);
    if (f != f) return 0xFFFFFFFFu;
    if (u == 0x80000000u) u = 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_float(uint32_t k) {
    uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(u);
}

// A score takes part in a top-k only if it could ever enter the reference's
// buffer, whose empty slots hold +inf and which replaces on a strict '<'
// (AgentMemory/M3/src/cluster.cpp:239-272): +inf and NaN never do.
__device__ __forceinline__ bool score_valid(float s) { return s < __int_as_float(0x7f800000); }

}  // namespace m3g
