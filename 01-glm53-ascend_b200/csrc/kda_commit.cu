// Speculative-decoding commit of the GLM KDA operator on sm_100a, behind
// kda_commit_intermediate_launch.
//
// After a verify pass the recurrent kernel has written one fp32 checkpoint per
// (request, draft step, head) into the caller's scratch. Committing the
// accepted step is a gather of D x D blocks into the pool:
//     dst[l, dst_indices[i], h] <- src[l, src_indices[i], step_indices[i], h]
// which sglang does with sgl_kernel_npu's move_intermediate_cache_kda (the
// call in sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:87-99;
// the function itself is not part of the reference tree).
//
// One CTA per (entry, layer, head) block: 64 KiB read + 64 KiB written at
// D = 128, so the kernel is HBM-bound and only needs wide, coalesced accesses.
// When both sides store the block densely in the same element order (the
// production pool and the recurrent kernel's scratch do), the block is one
// linear run copied in 16-byte pieces; any other strides take an element loop.

#include "kda_common.cuh"

#include <climits>

namespace kda {
namespace commit {

constexpr int kThreads = 256;

template <bool LINEAR>
__global__ void __launch_bounds__(kThreads) commit_kernel(const KdaCommitArgs p) {
    const int64_t item = blockIdx.x;
    const int h = static_cast<int>(item % p.num_heads);
    const int64_t rest = item / p.num_heads;
    const int l = static_cast<int>(rest % p.num_layers);
    const int64_t i = rest / p.num_layers;
    const int64_t slot = load_index(p.dst_indices, p.index_bytes[0], i);
    const int64_t req = load_index(p.src_indices, p.index_bytes[1], i);
    const int64_t step = load_index(p.step_indices, p.index_bytes[2], i);
    if (step < 0) return;   // nothing accepted for this entry
    if (slot < 0 || slot >= p.num_slots || req < 0 || req >= p.num_requests || step >= p.num_steps) {
        if (threadIdx.x == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
        return;
    }
    float *d = p.dst + l * p.dst_stride[0] + slot * p.dst_stride[1] + h * p.dst_stride[2];
    const float *s = p.src + l * p.src_stride[0] + req * p.src_stride[1] + step * p.src_stride[2] +
                     h * p.src_stride[3];
    const int D = p.head_dim;
    const int64_t n = static_cast<int64_t>(D) * D;
    if constexpr (LINEAR) {
        const float4 *s4 = reinterpret_cast<const float4 *>(s);
        float4 *d4 = reinterpret_cast<float4 *>(d);
        for (int64_t e = threadIdx.x; e < n / 4; e += kThreads) d4[e] = __ldcs(s4 + e);
    } else {
        const int64_t dr = p.dst_stride[3], dc = p.dst_stride[4];
        const int64_t sr = p.src_stride[4], sc = p.src_stride[5];
        for (int64_t e = threadIdx.x; e < n; e += kThreads) {
            const int64_t r = e / D, c = e % D;
            d[r * dr + c * dc] = s[r * sr + c * sc];
        }
    }
}

}  // namespace commit
}  // namespace kda

extern "C" int kda_commit_intermediate_launch(const KdaCommitArgs *args, void *stream) {
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    const KdaCommitArgs &a = *args;
    if (a.num_entries < 0 || a.num_layers < 0 || a.num_heads < 0 || a.head_dim < 0 || a.num_slots < 0 ||
        a.num_requests < 0 || a.num_steps < 0)
        return KDA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 3; ++i)
        if (a.index_bytes[i] != 4 && a.index_bytes[i] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (a.num_entries == 0 || a.num_layers == 0 || a.num_heads == 0 || a.head_dim == 0) return KDA_OK;
    if (a.dst == nullptr || a.src == nullptr || a.dst_indices == nullptr || a.src_indices == nullptr ||
        a.step_indices == nullptr)
        return KDA_ERR_INVALID_ARGUMENT;
    const int64_t blocks = static_cast<int64_t>(a.num_entries) * a.num_layers * a.num_heads;
    if (blocks > INT_MAX) return KDA_ERR_TOO_LARGE;

    // Linear path: both blocks dense in the same element order, and every
    // block base 16-byte aligned (base pointers aligned, outer strides
    // multiples of 4 elements, D * D a multiple of 4).
    const int64_t D = a.head_dim;
    const bool same_order = a.dst_stride[3] == a.src_stride[4] && a.dst_stride[4] == a.src_stride[5];
    const bool dense = (a.dst_stride[3] == D && a.dst_stride[4] == 1) || (a.dst_stride[3] == 1 && a.dst_stride[4] == D);
    bool aligned = (reinterpret_cast<uintptr_t>(a.dst) & 15u) == 0 && (reinterpret_cast<uintptr_t>(a.src) & 15u) == 0 &&
                   (D * D) % 4 == 0;
    for (int i = 0; i < 3; ++i) aligned = aligned && a.dst_stride[i] % 4 == 0;
    for (int i = 0; i < 4; ++i) aligned = aligned && a.src_stride[i] % 4 == 0;

    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (same_order && dense && aligned)
        kda::commit::commit_kernel<true><<<static_cast<unsigned>(blocks), kda::commit::kThreads, 0, st>>>(a);
    else
        kda::commit::commit_kernel<false><<<static_cast<unsigned>(blocks), kda::commit::kThreads, 0, st>>>(a);
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
