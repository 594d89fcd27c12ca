// Self-test of the bounded mbarrier wait (kda::mbar_wait) that every kernel of
// this library uses, behind kda_selftest_wait_timeout. No counterpart in the
// reference, whose waits (IBWait, kda_varlen_recurrent_prefill_h4.cpp:410-414)
// are unbounded.
//
// One CTA waits on an mbarrier that nothing ever arrives on, so every wait
// runs out of polls: it must record KDA_DEVICE_ERR_WAIT_TIMEOUT in the status
// word and return false, and the kernel must then end normally. With the
// CTA-wide give-up word, only the first expiry costs the full poll budget;
// later waits of the CTA give up at their first poll.

#include "kda_common.cuh"

namespace kda {

__global__ void __launch_bounds__(64) wait_selftest_kernel(int32_t *status, int32_t *expired, uint32_t polls,
                                                           int waits, int give_up) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int32_t abort_w;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_w = 0;
        fence_mbar_init();
    }
    __syncthreads();
    int n = 0;
    for (int i = 0; i < waits; ++i)
        if (!mbar_wait(&bar, 0u, status, give_up ? &abort_w : nullptr, polls)) ++n;
    if (n > 0) atomicAdd(expired, n);
}

}  // namespace kda

extern "C" int kda_selftest_wait_timeout(int32_t *status, int32_t *expired, int32_t polls, int32_t waits,
                                         int32_t give_up, void *stream) {
    if (status == nullptr || expired == nullptr || polls <= 0 || waits <= 0 || waits > 64) return KDA_ERR_INVALID_ARGUMENT;
    kda::wait_selftest_kernel<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(
        status, expired, static_cast<uint32_t>(polls), waits, give_up);
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
