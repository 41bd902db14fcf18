// tma_util.cuh -- TMA tensor maps, mbarriers and bounded waits shared by the
// TMA-fed kernels (the tcgen05 GEMM and the staged element-wise chain).
//
// Every TMA load here targets one CTA's own shared memory (no cluster-wide
// delivery): these kernels run on every rank of a multi-GPU job and only
// ever read this GPU's own memory.
#pragma once
#include <cuda.h>

#include "ttc_internal.cuh"

namespace ttc {

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
// dims / strides in elements of 4 bytes; strides[i] is the pitch of dim i+1.
int encode_tensor_map_f32(CUtensorMap* map, const void* ptr, int rank, const unsigned long long* dims,
                          const unsigned long long* strides_elems, const unsigned* box, CUtensorMapSwizzle swizzle);
// Host-mapped status word a kernel sets when one of its bounded waits expires.
int device_status_ptr(int** dptr);

constexpr long long kWaitLimitCycles = 4000000000ll;  // ~2 s at 1.9 GHz
// Failure-detection test switch, read at every launch: TTC_TEST_STALL=gemm
// (the TF32 GEMM kernels) or =chain (the TMA-staged chain kernel) makes the
// kernel's TMA producer issue no loads at all, so nothing is ever in flight
// and the consumers' waits run out after kStallTestLimitCycles (~1 ms); they
// set the status word, free what they hold and return, and the next
// synchronisation reports TTC_ERR_TIMEOUT. Returns whether `family` stalls.
constexpr long long kStallTestLimitCycles = 2000000ll;
bool stall_test(const char* family);

#ifdef __CUDACC__

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait for the phase with the given parity; false when it expired
// (after `limit` SM clock cycles).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long limit = kWaitLimitCycles) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > limit) return false;
    return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
        : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
        "[%2];" ::"r"(dst),
        "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}
__device__ __forceinline__ void prefetch_tensor_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}
// Barrier among `count` threads (a subset of the block) on hardware barrier `id`.
__device__ __forceinline__ void named_barrier(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
#endif

}  // namespace ttc
