// common.cuh -- sm_100a device helpers shared by the Q38RT B200 kernels:
// mbarrier pipelines, TMA bulk copies, programmatic dependent launch (PDL)
// and the bounded-wait fault word.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_fp16.h>

namespace q38 {

// Every spin in these kernels gives up after this many polls, records the
// site in the device fault word and lets the kernel return normally, so a
// lost TMA completion turns into an error status on the host instead of a
// hung GPU.  One poll of try_wait suspends for at most a few microseconds,
// so the bound is far above any legal wait and well below a second.
constexpr uint32_t kSpinLimit = 1u << 22;

enum FaultSite : uint32_t {
    kFaultNone = 0,
    kFaultFullWait = 1,   // consumer waited too long for a TMA tile
    kFaultEmptyWait = 2,  // producer waited too long for a free slot
    kFaultDrain = 3,      // producer could not drain its copies at exit
    kFaultShape = 4,      // kernel launched with an unsupported shape
    kFaultPeerWait = 5,   // tensor-parallel exchange: a peer's partial never arrived
};

// Written with atomicCAS so the first fault wins; read and cleared by the host
// through q38_fault_status() / q38_fault_clear().  The library is one CUDA
// translation unit (q38rt.cu includes every kernel header), so this
// definition exists exactly once.
__device__ uint32_t g_q38_fault;

__device__ __forceinline__ void record_fault(uint32_t site) {
    atomicCAS(&g_q38_fault, 0u, site);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
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

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded spin for data that is usually already there: a non-suspending test
// first, then the suspending try_wait.  False (fault recorded) when the poll
// budget runs out.
__device__ __forceinline__ bool mbar_wait_spin(uint64_t* bar, uint32_t parity, uint32_t site) {
    if (mbar_test_wait(bar, parity)) return true;
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    record_fault(site);
    return false;
}

// Bounded wait: true when the phase completed, false (fault recorded) when
// the poll budget ran out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t site) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
    }
    record_fault(site);
    return false;
}

// Orders this thread's earlier generic-proxy shared-memory accesses before
// later async-proxy (TMA) accesses to the same memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---- TMA: 1-D bulk copy global -> shared, completion on an mbarrier --------
// dst and src 16-byte aligned, bytes a multiple of 16 (checked by callers).
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// 2-D tiled tensor copy; c0 is the inner (contiguous) coordinate in elements
// of the tensor map's data type.  No multicast anywhere in this project.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t c0, int32_t c1,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Non-blocking hint to bring the 128-byte line holding p into L1.
__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// ---- programmatic dependent launch -----------------------------------------
// wait: block until the preceding grid in the stream has completed and its
// writes are visible.  Everything issued before it must not read data that
// the predecessor produces (here: only weights are touched before it).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// launch_dependents: allow the next grid in the stream to be scheduled now.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- small integer helpers ---------------------------------------------------
__device__ __forceinline__ uint32_t rotl(uint32_t v, uint32_t s) { return __funnelshift_l(v, v, s); }

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) {
    return __dp4a(static_cast<int>(a), static_cast<int>(b), c);
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xffffu)));
}

}  // namespace q38
