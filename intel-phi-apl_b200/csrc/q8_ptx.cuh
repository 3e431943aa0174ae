// q8_ptx.cuh: the sm_100a PTX this library's kernels are built from: mbarriers, 1-D bulk
// (TMA) copies, L2 cache policies, a bounded wait and the error word. Only plain
// single-CTA bulk loads from this GPU's own memory appear here.
#pragma once
#include <cstdint>

namespace q8 {

// Error bits a kernel ORs into the context's device error word (read back by the host).
enum : unsigned {
    ERR_TIMEOUT_FULL = 1u << 0,   // a stage's bulk copy never completed
    ERR_TIMEOUT_TFULL = 1u << 1,  // the partial sums of a stage never arrived
    ERR_TIMEOUT_TEMPTY = 1u << 2, // the chain never released a partial-sum buffer
    ERR_TIMEOUT_MMA = 1u << 3,    // a tensor-core stage never completed
    ERR_TIMEOUT_DRAIN = 1u << 4,  // copies in flight at exit never completed
    ERR_BAD_JOB = 1u << 5,        // a gather index outside the matrix (its y is NaN), or a job the kernel cannot run
    ERR_TIMEOUT_PEER = 1u << 6,   // a peer GPU's flag never arrived
    ERR_TIMEOUT_ROUND = 1u << 7,  // a chained round's dependency never completed
    ERR_TIMEOUT_GATE = 1u << 8,   // an opened round's x never landed (no rt_gemv_go)
};

// A spin of about this many SM clocks (~1 s at 2 GHz) is a hang, not a slow GPU.
constexpr long long WAIT_LIMIT_CYCLES = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes the initialised barriers visible to the async proxy (the bulk copies).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_shared() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// The slow path of mbar_wait, out of line: keeps the kernels' hot loops small.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (clock64() - t0 > WAIT_LIMIT_CYCLES)
            return false;
    }
    return true;
}

// Waits for the barrier's phase with this parity to complete; false after WAIT_LIMIT_CYCLES.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity);
}

// An L2 policy for data read once (the weights): evict first, so the small operands that every
// CTA re-reads (x) stay resident.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// 1-D bulk copy global -> this CTA's shared memory; completion counted in bytes on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Programmatic dependent launch: let the next kernel on the stream start its prologue now, and
// (in the next kernel) wait until the previous kernel has completed and its writes are visible.
// Both are no-ops when the kernel was not launched with programmatic stream serialization.
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// The error word: err[0] the bits; at err + 2 (8-byte aligned) a pointer, or null, to a word in
// mapped host memory that is set to 1 as well, so the host learns of an error without a copy.
__device__ __forceinline__ void report(unsigned *err, unsigned bits) {
    if (err) {
        atomicOr(err, bits);
        unsigned *mirror = *reinterpret_cast<unsigned *const volatile *>(err + 2);
        if (mirror)
            *reinterpret_cast<volatile unsigned *>(mirror) = 1u;
    }
}

}  // namespace q8
