// Device helpers shared by the KDA kernels: bf16 unpacking, index loads,
// mbarrier + bulk-TMA (cp.async.bulk) primitives with bounded waits.
//
// Every wait here gives up after a fixed number of polls and records
// KDA_DEVICE_ERR_WAIT_TIMEOUT in the caller's status word instead of spinning
// forever.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "kda_b200.h"

namespace kda {

constexpr float kNormEps = 1e-6f;   // inside the sqrt, kda_python.py:28-29
constexpr uint32_t kMaxWaitPolls = 1u << 22;
constexpr uint32_t kWaitSuspendNs = 1000;   // per poll; bounds a wait at ~4 s

__device__ __forceinline__ float bf16_lo(uint32_t x) { return __uint_as_float(x << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }

__device__ __forceinline__ float bf16_to_f(const void *p, int64_t i) {
    const uint16_t bits = reinterpret_cast<const uint16_t *>(p)[i];
    return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

// Four consecutive bf16 (8-byte aligned) -> float4.
__device__ __forceinline__ float4 load_bf16x4(const void *p, int64_t i) {
    const uint2 r = __ldg(reinterpret_cast<const uint2 *>(reinterpret_cast<const uint16_t *>(p) + i));
    return make_float4(bf16_lo(r.x), bf16_hi(r.x), bf16_lo(r.y), bf16_hi(r.y));
}

__device__ __forceinline__ float4 load_f32x4(const float *p, int64_t i) {
    return __ldg(reinterpret_cast<const float4 *>(p + i));
}

// int32 or int64 metadata, narrowed on read (an int64 buffer read as int32
// would alias high words; test_kda_index_dtypes.py:1-16 pins this).
__device__ __forceinline__ int64_t load_index(const void *p, int bytes, int64_t i) {
    if (bytes == 8) return reinterpret_cast<const int64_t *>(p)[i];
    return reinterpret_cast<const int32_t *>(p)[i];
}

__device__ __forceinline__ void report(int32_t *status, int32_t code) {
    if (status != nullptr) atomicCAS(status, 0, code);
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

// ---------------------------------------------------------------------------
// mbarrier + bulk copy (sm_90+ PTX; used on sm_100a)
// ---------------------------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
                 : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}

// One poll of an mbarrier phase. The suspend-time hint lets a waiting warp
// sleep instead of spinning, leaving issue slots to the warps that do the work.
__device__ __forceinline__ bool mbar_try(uint32_t addr, uint32_t phase) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(addr), "r"(phase), "r"(kWaitSuspendNs)
        : "memory");
    return done != 0;
}

// Waits for `phase` of `bar` for at most `polls` polls. Returns false (and
// records KDA_DEVICE_ERR_WAIT_TIMEOUT) if the phase did not complete.
// `abort`, when given, is a CTA-wide shared-memory word (zeroed at kernel
// start): the first wait of the CTA that expires sets it, and from then on
// every wait of the CTA that does not complete at its first poll gives up at
// once. A CTA whose wait expired therefore runs to its end (through its
// barriers, freeing its tensor memory) in about one wait's time instead of
// one expiry per remaining wait; its results are undefined and the status
// word says so.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t phase, int32_t *status,
                                          volatile int32_t *abort = nullptr, uint32_t polls = kMaxWaitPolls) {
    const uint32_t addr = smem_addr(bar);
    for (uint32_t i = 0; i < polls; ++i) {
        if (mbar_try(addr, phase)) return true;
        if (abort != nullptr && *abort != 0) return false;
    }
    if (abort != nullptr) *abort = 1;
    report(status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
    return false;
}

// Host side (kda_recurrent.cu): the recurrence over the requests whose length
// lies in [len_lo, len_hi]; the other requests are neither read nor written.
int recurrent_launch_range(const KdaArgs *args, int32_t len_lo, int32_t len_hi, cudaStream_t st);

// 1-D bulk copy global -> shared, completion counted on `bar` in bytes.
// Both addresses 16-byte aligned, bytes a multiple of 16. No multicast.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

}  // namespace kda
