// Host ops of the B200 KDA operator: validation, output/workspace allocation,
// dispatch to the C ABI (kda_b200.h), and registration under the reference's
// torch-op namespace `sgl_glm53_ascend` on the CUDA dispatch key.
//
// Schemas are the reference's, verbatim:
//   kda_varlen_recurrent  sgl-glm53-ascend-ops/csrc/kda/recurrent/kda_varlen_recurrent.cpp:257-264
//   kda_varlen_chunk      sgl-glm53-ascend-ops/csrc/kda/chunk/kda_varlen_chunk.cpp:195-202
//   prepared_recurrent    sgl-glm53-ascend-ops/csrc/kda/prepared_recurrent.cpp:715-721
//   *_v2                  sgl-glm53-ascend-ops/csrc/kda/recurrent_v2/kda_varlen_recurrent_v2.cpp:226-238
//                         and chunk_v2/kda_varlen_chunk_v2.cpp (aliases of the real ops here)
// plus two log-gate ops (`kda_varlen_recurrent_g`, `kda_varlen_chunk_g`) that
// take the fp32 log-decay g and beta directly, and the speculative-decoding
// commit `move_intermediate_cache_kda` (sgl_kernel_npu's function of that name,
// which the reference's MTP test calls after a verify), and the causal-conv
// front end `kda_causal_conv1d` that feeds q, k and v to the KDA ops.
//
// Error messages keep the reference's wording where a caller matches on it
// ("must be K-contiguous", "does not support", "expects ...",
// tests/integration/kda_ascendc_dispatch.py:52-58). Rules the reference had
// only because of its hardware are dropped: any head count, multi-sequence
// recurrent prefill, K = V in {64, 128}, and chunk lengths that are not
// multiples of 64 (so no device-to-host copy of cu_seqlens is needed and the
// chunk op is CUDA-graph capturable).

#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <mutex>
#include <unordered_map>
#include <utility>

#include "kda_b200.h"

namespace {

using NamedTensor = std::pair<const char *, const at::Tensor &>;

// Optional per-device status word registered by the caller (tests); null
// otherwise. Never allocated here, so every op stays capture-safe.
std::mutex g_status_mu;
std::unordered_map<int, at::Tensor> g_status;

int32_t *status_ptr(const at::Device &dev) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    auto it = g_status.find(dev.index());
    return it == g_status.end() ? nullptr : it->second.data_ptr<int32_t>();
}

void check_kda(int rc, const char *op) {
    TORCH_CHECK(rc == KDA_OK, op, ": kernel launch rejected: ", kda_status_string(rc), " (", rc, ")");
}

int index_bytes(const at::Tensor &t) { return t.scalar_type() == at::kLong ? 8 : 4; }

void check_index(const char *name, const at::Tensor &t, const at::Tensor &q) {
    TORCH_CHECK(t.scalar_type() == at::kInt || t.scalar_type() == at::kLong, name,
                " must be int32 or int64");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
    TORCH_CHECK(t.device() == q.device(), name, " must be on the same device as q");
}

// Shared validation of the raw-gate and log-gate varlen ops (the reference's
// kda_varlen_recurrent.cpp:36-74, 111-122 and kda_varlen_chunk.cpp:35-105).
struct Dims {
    int64_t H, D, T, num_req;
};

Dims check_varlen(const char *op, const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                  std::initializer_list<NamedTensor> bf16_extra, at::Tensor &state,
                  const at::Tensor &indices, const at::Tensor &cu_seqlens,
                  const c10::optional<at::Tensor> &track_indices,
                  const c10::optional<at::Tensor> &track_lens) {
    TORCH_CHECK(q.is_cuda(), "q must be a CUDA tensor");
    for (const auto &named : {NamedTensor{"q", q}, NamedTensor{"k", k}, NamedTensor{"v", v}}) {
        TORCH_CHECK(named.second.scalar_type() == at::kBFloat16, named.first, " must be bf16");
        TORCH_CHECK(named.second.is_contiguous(), named.first, " must be contiguous");
        TORCH_CHECK(named.second.device() == q.device(), named.first, " must be on the same device as q");
    }
    for (const auto &named : bf16_extra) {
        TORCH_CHECK(named.second.scalar_type() == at::kBFloat16, named.first, " must be bf16");
        TORCH_CHECK(named.second.is_contiguous(), named.first, " must be contiguous");
        TORCH_CHECK(named.second.device() == q.device(), named.first, " must be on the same device as q");
    }
    TORCH_CHECK(q.dim() == 4 && k.dim() == 4 && v.dim() == 4 && q.size(0) == 1,
                op, " expects [1,T,H,D] q/k/v");
    const int64_t H = k.size(2), D = k.size(3), HV = v.size(2), DV = v.size(3);
    TORCH_CHECK(H == HV, op, " requires H == HV, got ", H, " and ", HV);
    TORCH_CHECK(D == DV && (D == 64 || D == 128), op, " requires K == V in {64, 128}, got ", D, " and ", DV);
    TORCH_CHECK(q.sizes() == k.sizes() && v.size(1) == q.size(1), op, " q/k/v token dimensions must match");
    TORCH_CHECK(state.dim() == 4 && state.scalar_type() == at::kFloat,
                "state must be a 4-D fp32 [slots,HV,K,V] pool");
    TORCH_CHECK(state.size(1) == HV && state.size(2) == D && state.size(3) == D,
                "state must be [slots,HV,K,V] matching the head and feature dims");
    TORCH_CHECK(state.stride(2) == 1 && state.stride(3) == D, "state must be K-contiguous (stride(2)==1, stride(3)==",
                D, "), got strides (", state.stride(2), ", ", state.stride(3), ")");
    TORCH_CHECK(state.device() == q.device(), "state must be on the same device as q");
    check_index("initial_state_indices", indices, q);
    check_index("cu_seqlens", cu_seqlens, q);
    const int64_t num_req = indices.numel();
    TORCH_CHECK(cu_seqlens.numel() == num_req + 1, "cu_seqlens must have numReq+1 entries, got ",
                cu_seqlens.numel(), " for ", num_req, " requests");
    if (track_indices.has_value()) {
        TORCH_CHECK(track_lens.has_value(), "track_state_indices requires track_state_lens");
        for (const auto &named : {NamedTensor{"track_state_indices", *track_indices},
                                  NamedTensor{"track_state_lens", *track_lens}}) {
            check_index(named.first, named.second, q);
            TORCH_CHECK(named.second.numel() == num_req, named.first, " must have one entry per request");
        }
    } else {
        TORCH_CHECK(!track_lens.has_value(), "track_state_lens requires track_state_indices");
    }
    return Dims{H, D, q.size(1), num_req};
}

KdaArgs base_args(const Dims &d, const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                  at::Tensor &out, at::Tensor &state, const at::Tensor &indices,
                  const at::Tensor &cu_seqlens, const c10::optional<at::Tensor> &track_indices,
                  const c10::optional<at::Tensor> &track_lens, double scale) {
    KdaArgs a{};
    a.q = q.data_ptr();
    a.k = k.data_ptr();
    a.v = v.data_ptr();
    a.out = out.data_ptr();
    a.state = state.data_ptr<float>();
    for (int i = 0; i < 4; ++i) a.state_stride[i] = state.stride(i);
    a.num_slots = state.size(0);
    a.indices = indices.data_ptr();
    a.cu_seqlens = cu_seqlens.data_ptr();
    a.index_bytes[0] = index_bytes(indices);
    a.index_bytes[1] = index_bytes(cu_seqlens);
    a.index_bytes[2] = track_indices.has_value() ? index_bytes(*track_indices) : 4;
    a.index_bytes[3] = track_lens.has_value() ? index_bytes(*track_lens) : 4;
    a.track_indices = track_indices.has_value() ? track_indices->data_ptr() : nullptr;
    a.track_lens = track_lens.has_value() ? track_lens->data_ptr() : nullptr;
    a.num_req = static_cast<int32_t>(d.num_req);
    a.num_tokens = static_cast<int32_t>(d.T);
    a.num_heads = static_cast<int32_t>(d.H);
    a.head_dim = static_cast<int32_t>(d.D);
    a.head_begin = 0;
    a.head_count = static_cast<int32_t>(d.H);
    a.scale = static_cast<float>(scale);
    a.status = status_ptr(q.device());
    return a;
}

void check_raw_gate(const char *op, const at::Tensor &A_log, const at::Tensor &dt_bias, const at::Tensor &b,
                    const at::Tensor &a, const Dims &d, const at::Tensor &q) {
    TORCH_CHECK(A_log.scalar_type() == at::kFloat && A_log.numel() == d.H, "A_log must be fp32 with HV elements");
    TORCH_CHECK(dt_bias.scalar_type() == at::kFloat && dt_bias.numel() == d.H * d.D,
                "dt_bias must be fp32 with HV*K elements");
    TORCH_CHECK(A_log.is_contiguous() && dt_bias.is_contiguous(), op, " A_log and dt_bias must be contiguous");
    TORCH_CHECK(A_log.device() == q.device() && dt_bias.device() == q.device(),
                "A_log and dt_bias must be on the same device as q");
    TORCH_CHECK(a.sizes() == q.sizes(), "a must have shape [1,T,HV,K]");
    TORCH_CHECK(b.dim() == 3 && b.size(1) == d.T && b.size(2) == d.H, "b must have shape [1,T,HV]");
}

void check_log_gate(const at::Tensor &g, const at::Tensor &beta, const Dims &d, const at::Tensor &q) {
    TORCH_CHECK(g.scalar_type() == at::kFloat && g.is_contiguous() && g.sizes() == q.sizes(),
                "g must be a contiguous fp32 [1,T,HV,K] tensor");
    TORCH_CHECK(beta.scalar_type() == at::kFloat && beta.is_contiguous() && beta.numel() == d.T * d.H,
                "beta must be a contiguous fp32 [1,T,HV] tensor");
    TORCH_CHECK(g.device() == q.device() && beta.device() == q.device(), "g and beta must be on the same device as q");
}

// intermediate_state rules (kda_varlen_recurrent.cpp:82-110).
void check_intermediate(const at::Tensor &mid, const Dims &d, const at::Tensor &q) {
    TORCH_CHECK(mid.dim() == 5 && mid.scalar_type() == at::kFloat,
                "intermediate_state must be a 5-D fp32 [slots,steps,HV,K,V] buffer");
    TORCH_CHECK(mid.size(2) == d.H && mid.size(3) == d.D && mid.size(4) == d.D,
                "intermediate_state must be [slots,steps,HV,K,V] matching the head and feature dims");
    TORCH_CHECK(mid.stride(3) == 1 && mid.stride(4) == d.D, "intermediate_state must be K-contiguous (stride(3)==1, "
                "stride(4)==", d.D, "), got strides (", mid.stride(3), ", ", mid.stride(4), ")");
    TORCH_CHECK(mid.device() == q.device(), "intermediate_state must be on the same device as q");
    TORCH_CHECK(mid.size(0) >= d.num_req, "intermediate_state needs a row per request, got ", mid.size(0), " for ",
                d.num_req, " requests");
    TORCH_CHECK(mid.size(1) * d.num_req >= d.T, "intermediate_state has ", mid.size(1), " step rows, too few for ",
                d.T, " tokens across ", d.num_req, " requests");
}

// Regime rules of the recurrent op (kda_varlen_recurrent.cpp:219-251) that
// are semantics rather than hardware limits.
void check_regime(const char *op, const Dims &d, bool prefill, bool save_intermediate, bool track) {
    if (prefill) {
        TORCH_CHECK(!save_intermediate, op, " prefill does not support intermediate_state");
    } else {
        TORCH_CHECK(d.T >= d.num_req, op, " decode expects at least one token per request, got T=", d.T,
                    " and numReq=", d.num_req);
        TORCH_CHECK(!track, op, " tracking is prefill-only");
    }
}

void set_intermediate(KdaArgs &a, const c10::optional<at::Tensor> &mid) {
    if (!mid.has_value()) return;
    a.intermediate = mid->data_ptr<float>();
    for (int i = 0; i < 5; ++i) a.mid_stride[i] = mid->stride(i);
}

cudaStream_t current_stream(const at::Tensor &q) { return at::cuda::getCurrentCUDAStream(q.device().index()).stream(); }

void launch_chunk(KdaArgs &a, const at::Tensor &v) {
    const size_t ws_bytes = kda_chunk_workspace_bytes(a.num_req, a.num_tokens, a.head_count, a.head_dim);
    at::Tensor ws = at::empty({static_cast<int64_t>(ws_bytes > 0 ? ws_bytes : 1)}, v.options().dtype(at::kByte));
    check_kda(kda_chunk_launch(&a, ws.data_ptr(), ws_bytes, current_stream(v)), "kda_varlen_chunk");
}

}  // namespace

at::Tensor kda_varlen_recurrent(const at::Tensor &A_log, const at::Tensor &a, const at::Tensor &dt_bias,
                                const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, const at::Tensor &b,
                                at::Tensor &initial_state_source, const at::Tensor &initial_state_indices,
                                const at::Tensor &cu_seqlens, double lower_bound, double scale,
                                const c10::optional<at::Tensor> &intermediate_state, bool prefill,
                                const c10::optional<at::Tensor> &track_state_indices,
                                const c10::optional<at::Tensor> &track_state_lens) {
    const char *op = "kda_varlen_recurrent";
    const Dims d = check_varlen(op, q, k, v, {NamedTensor{"a", a}, NamedTensor{"b", b}}, initial_state_source,
                                initial_state_indices, cu_seqlens, track_state_indices, track_state_lens);
    check_raw_gate(op, A_log, dt_bias, b, a, d, q);
    if (intermediate_state.has_value()) check_intermediate(*intermediate_state, d, q);
    check_regime(op, d, prefill, intermediate_state.has_value(), track_state_indices.has_value());
    c10::cuda::CUDAGuard guard(q.device());
    // The reference returns zeros_like(v) (kda_varlen_recurrent.cpp:142); the
    // kernel writes zeros itself wherever it computes no value (tokens no
    // request covers, rejected requests), which saves a separate fill.
    at::Tensor out = d.num_req > 0 ? at::empty_like(v) : at::zeros_like(v);
    KdaArgs args = base_args(d, q, k, v, out, initial_state_source, initial_state_indices, cu_seqlens,
                             track_state_indices, track_state_lens, scale);
    args.gate_mode = KDA_GATE_RAW;
    args.a = a.data_ptr();
    args.b = b.data_ptr();
    args.A_log = A_log.data_ptr<float>();
    args.dt_bias = dt_bias.data_ptr<float>();
    args.lower_bound = static_cast<float>(lower_bound);
    set_intermediate(args, intermediate_state);
    check_kda(kda_recurrent_launch(&args, current_stream(q)), op);
    return out;
}

at::Tensor kda_varlen_chunk(const at::Tensor &A_log, const at::Tensor &a, const at::Tensor &dt_bias,
                            const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, const at::Tensor &b,
                            at::Tensor &initial_state_source, const at::Tensor &initial_state_indices,
                            const at::Tensor &cu_seqlens, double lower_bound, double scale, bool prefill,
                            const c10::optional<at::Tensor> &track_state_indices,
                            const c10::optional<at::Tensor> &track_state_lens) {
    (void)prefill;  // accepted and unused, as in kda_varlen_chunk.cpp:25
    const char *op = "kda_varlen_chunk";
    const Dims d = check_varlen(op, q, k, v, {NamedTensor{"a", a}, NamedTensor{"b", b}}, initial_state_source,
                                initial_state_indices, cu_seqlens, track_state_indices, track_state_lens);
    check_raw_gate(op, A_log, dt_bias, b, a, d, q);
    c10::cuda::CUDAGuard guard(q.device());
    at::Tensor out = at::empty_like(v);
    KdaArgs args = base_args(d, q, k, v, out, initial_state_source, initial_state_indices, cu_seqlens,
                             track_state_indices, track_state_lens, scale);
    args.gate_mode = KDA_GATE_RAW;
    args.a = a.data_ptr();
    args.b = b.data_ptr();
    args.A_log = A_log.data_ptr<float>();
    args.dt_bias = dt_bias.data_ptr<float>();
    args.lower_bound = static_cast<float>(lower_bound);
    launch_chunk(args, v);
    return out;
}

at::Tensor kda_varlen_recurrent_g(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v,
                                  const at::Tensor &g, const at::Tensor &beta, at::Tensor &initial_state_source,
                                  const at::Tensor &initial_state_indices, const at::Tensor &cu_seqlens,
                                  double scale, const c10::optional<at::Tensor> &intermediate_state, bool prefill,
                                  const c10::optional<at::Tensor> &track_state_indices,
                                  const c10::optional<at::Tensor> &track_state_lens) {
    const char *op = "kda_varlen_recurrent_g";
    const Dims d = check_varlen(op, q, k, v, {}, initial_state_source, initial_state_indices, cu_seqlens,
                                track_state_indices, track_state_lens);
    check_log_gate(g, beta, d, q);
    if (intermediate_state.has_value()) check_intermediate(*intermediate_state, d, q);
    check_regime(op, d, prefill, intermediate_state.has_value(), track_state_indices.has_value());
    c10::cuda::CUDAGuard guard(q.device());
    // The reference returns zeros_like(v) (kda_varlen_recurrent.cpp:142); the
    // kernel writes zeros itself wherever it computes no value (tokens no
    // request covers, rejected requests), which saves a separate fill.
    at::Tensor out = d.num_req > 0 ? at::empty_like(v) : at::zeros_like(v);
    KdaArgs args = base_args(d, q, k, v, out, initial_state_source, initial_state_indices, cu_seqlens,
                             track_state_indices, track_state_lens, scale);
    args.gate_mode = KDA_GATE_LOG;
    args.g = g.data_ptr<float>();
    args.beta = beta.data_ptr<float>();
    set_intermediate(args, intermediate_state);
    check_kda(kda_recurrent_launch(&args, current_stream(q)), op);
    return out;
}

at::Tensor kda_varlen_chunk_g(const at::Tensor &q, const at::Tensor &k, const at::Tensor &v, const at::Tensor &g,
                              const at::Tensor &beta, at::Tensor &initial_state_source,
                              const at::Tensor &initial_state_indices, const at::Tensor &cu_seqlens, double scale,
                              bool prefill, const c10::optional<at::Tensor> &track_state_indices,
                              const c10::optional<at::Tensor> &track_state_lens) {
    (void)prefill;
    const char *op = "kda_varlen_chunk_g";
    const Dims d = check_varlen(op, q, k, v, {}, initial_state_source, initial_state_indices, cu_seqlens,
                                track_state_indices, track_state_lens);
    check_log_gate(g, beta, d, q);
    c10::cuda::CUDAGuard guard(q.device());
    at::Tensor out = at::empty_like(v);
    KdaArgs args = base_args(d, q, k, v, out, initial_state_source, initial_state_indices, cu_seqlens,
                             track_state_indices, track_state_lens, scale);
    args.gate_mode = KDA_GATE_LOG;
    args.g = g.data_ptr<float>();
    args.beta = beta.data_ptr<float>();
    launch_chunk(args, v);
    return out;
}

// prepared_recurrent (prepared_recurrent.cpp:610-713): heads [head_offset,
// head_offset + 4) of every request, on fp32 qn/kn/gdecay/beta; `out` and
// `state` are written in place.
void prepared_recurrent(const at::Tensor &qn, const at::Tensor &kn, const at::Tensor &v, const at::Tensor &gdecay,
                        const at::Tensor &beta, at::Tensor &out, at::Tensor &state, const at::Tensor &indices,
                        const at::Tensor &starts, const c10::optional<at::Tensor> &track_indices,
                        const c10::optional<at::Tensor> &track_lens, bool track_state, int64_t head_offset) {
    TORCH_CHECK(qn.is_cuda(), "qn must be a CUDA tensor");
    TORCH_CHECK(kn.is_cuda(), "kn must be a CUDA tensor");
    TORCH_CHECK(v.is_cuda(), "v must be a CUDA tensor");
    constexpr int64_t kHeadsPerLaunch = 4;
    TORCH_CHECK(state.dim() == 4 && state.scalar_type() == at::kFloat && state.size(2) == state.size(3),
                "state must be a 4-D fp32 [slots,H,D,D] pool");
    const int64_t H = state.size(1), D = state.size(2);
    TORCH_CHECK(D == 64 || D == 128, "prepared_recurrent supports D in {64, 128}, got ", D);
    TORCH_CHECK(head_offset >= 0 && head_offset < H, "head_offset must be in [0, ", H, "), got ", head_offset);
    for (const auto &named : {NamedTensor{"qn", qn}, NamedTensor{"kn", kn}, NamedTensor{"gdecay", gdecay},
                              NamedTensor{"beta", beta}}) {
        TORCH_CHECK(named.second.scalar_type() == at::kFloat, named.first, " must be fp32");
        TORCH_CHECK(named.second.is_contiguous(), named.first, " must be contiguous");
        TORCH_CHECK(named.second.device() == qn.device(), named.first, " must be on the same device as qn");
    }
    for (const auto &named : {NamedTensor{"v", v}, NamedTensor{"out", out}}) {
        TORCH_CHECK(named.second.scalar_type() == at::kBFloat16, named.first, " must be bf16");
        TORCH_CHECK(named.second.is_contiguous(), named.first, " must be contiguous");
        TORCH_CHECK(named.second.device() == qn.device(), named.first, " must be on the same device as qn");
    }
    const int64_t T = qn.numel() / (H * D);
    TORCH_CHECK(T * H * D == qn.numel() && kn.numel() == qn.numel() && gdecay.numel() == qn.numel() &&
                    v.numel() == qn.numel() && out.numel() == qn.numel() && beta.numel() == T * H,
                "prepared_recurrent expects qn/kn/gdecay/v/out of T*H*D elements and beta of T*H");
    check_index("indices", indices, qn);
    check_index("starts", starts, qn);
    const int64_t num_req = indices.numel();
    TORCH_CHECK(starts.numel() >= num_req + 1, "starts must have numReq+1 entries");
    const void *tidx = nullptr, *tlen = nullptr;
    int tib = 4, tlb = 4;
    if (track_state) {
        TORCH_CHECK(track_indices.has_value() && track_indices->defined(),
                    "track_indices is required when track_state=True");
        TORCH_CHECK(track_lens.has_value() && track_lens->defined(), "track_lens is required when track_state=True");
        for (const auto &named : {NamedTensor{"track_indices", *track_indices}, NamedTensor{"track_lens", *track_lens}}) {
            TORCH_CHECK(named.second.device() == qn.device(), named.first, " must be on the same device as qn");
            TORCH_CHECK(named.second.scalar_type() == at::kInt || named.second.scalar_type() == at::kLong,
                        named.first, " must be int32 or int64");
            TORCH_CHECK(named.second.is_contiguous(), named.first, " must be contiguous");
            TORCH_CHECK(named.second.numel() >= num_req, named.first, " must contain at least ", num_req,
                        " elements");
        }
        tidx = track_indices->data_ptr();
        tlen = track_lens->data_ptr();
        tib = index_bytes(*track_indices);
        tlb = index_bytes(*track_lens);
    }
    c10::cuda::CUDAGuard guard(qn.device());
    KdaArgs a{};
    a.q = qn.data_ptr();
    a.k = kn.data_ptr();
    a.v = v.data_ptr();
    a.g = gdecay.data_ptr<float>();
    a.beta = beta.data_ptr<float>();
    a.out = out.data_ptr();
    a.state = state.data_ptr<float>();
    for (int i = 0; i < 4; ++i) a.state_stride[i] = state.stride(i);
    a.num_slots = state.size(0);
    a.indices = indices.data_ptr();
    a.cu_seqlens = starts.data_ptr();
    a.track_indices = tidx;
    a.track_lens = tlen;
    a.index_bytes[0] = index_bytes(indices);
    a.index_bytes[1] = index_bytes(starts);
    a.index_bytes[2] = tib;
    a.index_bytes[3] = tlb;
    a.num_req = static_cast<int32_t>(num_req);
    a.num_tokens = static_cast<int32_t>(T);
    a.num_heads = static_cast<int32_t>(H);
    a.head_dim = static_cast<int32_t>(D);
    a.head_begin = static_cast<int32_t>(head_offset);
    a.head_count = static_cast<int32_t>(std::min<int64_t>(kHeadsPerLaunch, H - head_offset));
    a.gate_mode = KDA_GATE_PREPARED;
    a.status = status_ptr(qn.device());
    check_kda(kda_prepared_recurrent_launch(&a, current_stream(qn)), "prepared_recurrent");
}

// move_intermediate_cache_kda: the speculative-decoding commit, called as
// sgl_kernel_npu's function of that name is at
// sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:93-99:
//   dst [layers, slots, H, D, D] (in place) <- src [layers, requests, steps, H, D, D]
// entry i: dst[:, dst_indices[i]] = src[:, src_indices[i], step_indices[i]].
// `h_block_size` is the original's heads-per-program tiling; it does not change
// the result and is only range-checked.
void move_intermediate_cache_kda(at::Tensor &dst, const at::Tensor &src, const at::Tensor &dst_indices,
                                 const at::Tensor &src_indices, const at::Tensor &step_indices,
                                 int64_t h_block_size) {
    TORCH_CHECK(dst.is_cuda(), "dst must be a CUDA tensor");
    TORCH_CHECK(src.device() == dst.device(), "src must be on the same device as dst");
    TORCH_CHECK(dst.scalar_type() == at::kFloat && src.scalar_type() == at::kFloat, "dst and src must be fp32");
    TORCH_CHECK(dst.dim() == 5, "dst must be [layers, slots, H, D, D], got ", dst.dim(), " dims");
    TORCH_CHECK(src.dim() == 6, "src must be [layers, requests, steps, H, D, D], got ", src.dim(), " dims");
    TORCH_CHECK(dst.size(3) == dst.size(4) && src.size(4) == dst.size(3) && src.size(5) == dst.size(4),
                "dst and src must hold D x D blocks of the same D");
    TORCH_CHECK(src.size(0) == dst.size(0) && src.size(3) == dst.size(2),
                "dst and src must have the same layers and heads");
    TORCH_CHECK(h_block_size >= 1, "h_block_size must be positive");
    check_index("dst_indices", dst_indices, dst);
    check_index("src_indices", src_indices, dst);
    check_index("step_indices", step_indices, dst);
    const int64_t n = dst_indices.numel();
    TORCH_CHECK(src_indices.numel() == n && step_indices.numel() == n,
                "dst_indices, src_indices and step_indices must have the same length");
    c10::cuda::CUDAGuard guard(dst.device());
    KdaCommitArgs a{};
    a.dst = dst.data_ptr<float>();
    a.src = src.data_ptr<float>();
    for (int i = 0; i < 5; ++i) a.dst_stride[i] = dst.stride(i);
    for (int i = 0; i < 6; ++i) a.src_stride[i] = src.stride(i);
    a.dst_indices = dst_indices.data_ptr();
    a.src_indices = src_indices.data_ptr();
    a.step_indices = step_indices.data_ptr();
    a.index_bytes[0] = index_bytes(dst_indices);
    a.index_bytes[1] = index_bytes(src_indices);
    a.index_bytes[2] = index_bytes(step_indices);
    a.num_entries = static_cast<int32_t>(n);
    a.num_layers = static_cast<int32_t>(dst.size(0));
    a.num_heads = static_cast<int32_t>(dst.size(2));
    a.head_dim = static_cast<int32_t>(dst.size(3));
    a.num_slots = dst.size(1);
    a.num_requests = static_cast<int32_t>(src.size(1));
    a.num_steps = static_cast<int32_t>(src.size(2));
    a.status = status_ptr(dst.device());
    check_kda(kda_commit_intermediate_launch(&a, current_stream(dst)), "move_intermediate_cache_kda");
}

// kda_causal_conv1d: the causal-conv front end of the attention layer
// (kda_conv_launch), the causal_conv1d step sglang's backend runs on the mixed
// q | k | v projection before the KDA op
// (sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387):
//   x          [T, C] or [1, T, C] bf16, channels contiguous (a column slice of
//              a wider projection is fine: any row stride that is a multiple of 8)
//   weight     [C, W] (W <= 4; any float dtype, used as fp32), bias [C] or None
//   conv_state [slots, window, C] bf16, updated in place (W - 1 <= window <= 8)
//   cache_indices [R], query_start_loc [R + 1]: int32 or int64
//   has_initial_state [R] bool/int or None (None: every request continues)
//   track_conv_indices, track_conv_lens [R] or None: tracked-prefix checkpoint
// Returns [num_parts, T, C / num_parts] bf16: with num_parts = 3 the q, k and v
// planes, each the contiguous [T, H, D] tensor the KDA op takes.
at::Tensor kda_causal_conv1d(const at::Tensor &x, const at::Tensor &weight, const c10::optional<at::Tensor> &bias,
                             at::Tensor &conv_state, const at::Tensor &cache_indices,
                             const at::Tensor &query_start_loc, const c10::optional<at::Tensor> &has_initial_state,
                             const c10::optional<at::Tensor> &track_conv_indices,
                             const c10::optional<at::Tensor> &track_conv_lens, int64_t num_parts, bool silu) {
    TORCH_CHECK(x.is_cuda(), "x must be a CUDA tensor");
    TORCH_CHECK(x.scalar_type() == at::kBFloat16, "x must be bf16");
    TORCH_CHECK(x.dim() == 2 || (x.dim() == 3 && x.size(0) == 1), "kda_causal_conv1d expects [T, C] or [1, T, C] x");
    const at::Tensor x2 = x.dim() == 3 ? x.select(0, 0) : x;
    TORCH_CHECK(x2.stride(1) == 1, "x must be channel-contiguous (stride(-1) == 1)");
    const int64_t T = x2.size(0), C = x2.size(1);
    TORCH_CHECK(weight.dim() == 2 && weight.size(0) == C, "weight must be [C, W] with C = ", C);
    const int64_t W = weight.size(1);
    TORCH_CHECK(W >= 1 && W <= 4, "kda_causal_conv1d does not support ", W, " taps (1..4)");
    TORCH_CHECK(weight.device() == x.device(), "weight must be on the same device as x");
    const at::Tensor w32 = weight.to(at::kFloat).contiguous();
    at::Tensor b32;
    if (bias.has_value() && bias->defined()) {
        TORCH_CHECK(bias->numel() == C && bias->device() == x.device(), "bias must be [C] on the device of x");
        b32 = bias->to(at::kFloat).contiguous();
    }
    TORCH_CHECK(conv_state.dim() == 3 && conv_state.scalar_type() == at::kBFloat16 && conv_state.size(2) == C,
                "conv_state must be a bf16 [slots, window, C] tensor with C = ", C);
    TORCH_CHECK(conv_state.stride(2) == 1, "conv_state must be channel-contiguous (stride(2) == 1)");
    TORCH_CHECK(conv_state.device() == x.device(), "conv_state must be on the same device as x");
    TORCH_CHECK(conv_state.size(1) >= W - 1, "conv_state window (", conv_state.size(1), ") must hold W - 1 = ",
                W - 1, " rows");
    TORCH_CHECK(num_parts >= 1 && C % num_parts == 0, "num_parts must divide C");
    check_index("cache_indices", cache_indices, x);
    check_index("query_start_loc", query_start_loc, x);
    const int64_t R = cache_indices.numel();
    TORCH_CHECK(query_start_loc.numel() == R + 1, "query_start_loc must have len(cache_indices) + 1 entries");
    TORCH_CHECK(track_conv_indices.has_value() == track_conv_lens.has_value(),
                "track_conv_indices and track_conv_lens must be given together");
    if (track_conv_indices.has_value()) {
        check_index("track_conv_indices", *track_conv_indices, x);
        check_index("track_conv_lens", *track_conv_lens, x);
        TORCH_CHECK(track_conv_indices->numel() == R && track_conv_lens->numel() == R,
                    "track_conv_indices and track_conv_lens must have one entry per request");
    }
    int32_t init_bytes = 1;
    if (has_initial_state.has_value()) {
        const auto &hi = *has_initial_state;
        TORCH_CHECK(hi.numel() == R && hi.is_contiguous() && hi.device() == x.device(),
                    "has_initial_state must be a contiguous [R] tensor on the device of x");
        TORCH_CHECK(hi.scalar_type() == at::kBool || hi.scalar_type() == at::kByte || hi.scalar_type() == at::kInt ||
                        hi.scalar_type() == at::kLong,
                    "has_initial_state must be bool, uint8, int32 or int64");
        init_bytes = static_cast<int32_t>(hi.element_size());
    }
    c10::cuda::CUDAGuard guard(x.device());
    at::Tensor out = at::empty({num_parts, T, C / num_parts}, x.options());
    KdaConvArgs a{};
    a.x = x2.data_ptr();
    a.x_row_stride = x2.stride(0);
    a.weight = w32.data_ptr<float>();
    a.bias = b32.defined() ? b32.data_ptr<float>() : nullptr;
    a.conv_state = conv_state.data_ptr();
    a.state_stride[0] = conv_state.stride(0);
    a.state_stride[1] = conv_state.stride(1);
    a.num_slots = conv_state.size(0);
    a.window = static_cast<int32_t>(conv_state.size(1));
    a.indices = cache_indices.data_ptr();
    a.cu_seqlens = query_start_loc.data_ptr();
    a.has_initial = has_initial_state.has_value() ? has_initial_state->data_ptr() : nullptr;
    a.track_indices = track_conv_indices.has_value() ? track_conv_indices->data_ptr() : nullptr;
    a.track_lens = track_conv_lens.has_value() ? track_conv_lens->data_ptr() : nullptr;
    a.index_bytes[0] = index_bytes(cache_indices);
    a.index_bytes[1] = index_bytes(query_start_loc);
    a.index_bytes[2] = init_bytes;
    a.index_bytes[3] = track_conv_indices.has_value() ? index_bytes(*track_conv_indices) : 4;
    a.index_bytes[4] = track_conv_lens.has_value() ? index_bytes(*track_conv_lens) : 4;
    a.num_req = static_cast<int32_t>(R);
    a.num_tokens = static_cast<int32_t>(T);
    a.channels = static_cast<int32_t>(C);
    a.width = static_cast<int32_t>(W);
    a.num_parts = static_cast<int32_t>(num_parts);
    a.activation = silu ? KDA_CONV_ACT_SILU : KDA_CONV_ACT_NONE;
    a.out = out.data_ptr();
    a.status = status_ptr(x.device());
    check_kda(kda_conv_launch(&a, current_stream(x)), "kda_causal_conv1d");
    return out;
}

// Registers (or clears, with an undefined tensor) an int32 device word that
// the kernels on that device report KDA_DEVICE_ERR_* codes into.
void kda_set_status_buffer(int64_t device, const c10::optional<at::Tensor> &buf) {
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (!buf.has_value() || !buf->defined()) {
        g_status.erase(static_cast<int>(device));
        return;
    }
    TORCH_CHECK(buf->is_cuda() && buf->scalar_type() == at::kInt && buf->numel() >= 1,
                "status buffer must be a CUDA int32 tensor");
    g_status[static_cast<int>(device)] = *buf;
}

int64_t kda_abi_version_op() { return kda_abi_version(); }

TORCH_LIBRARY(sgl_glm53_ascend, m) {
    const char *recurrent_schema =
        "(*, Tensor A_log, Tensor a, Tensor dt_bias, Tensor q, Tensor k, Tensor v, Tensor b, "
        "Tensor(a!) initial_state_source, Tensor initial_state_indices, Tensor cu_seqlens, "
        "float lower_bound, float scale, Tensor(b!)? intermediate_state=None, bool prefill=False, "
        "Tensor? track_state_indices=None, Tensor? track_state_lens=None) -> Tensor";
    const char *chunk_schema =
        "(*, Tensor A_log, Tensor a, Tensor dt_bias, Tensor q, Tensor k, Tensor v, Tensor b, "
        "Tensor(a!) initial_state_source, Tensor initial_state_indices, Tensor cu_seqlens, "
        "float lower_bound, float scale, bool prefill=False, Tensor? track_state_indices=None, "
        "Tensor? track_state_lens=None) -> Tensor";
    m.def((std::string("kda_varlen_recurrent") + recurrent_schema).c_str());
    m.def((std::string("kda_varlen_recurrent_v2") + recurrent_schema).c_str());
    m.def((std::string("kda_varlen_chunk") + chunk_schema).c_str());
    m.def((std::string("kda_varlen_chunk_v2") + chunk_schema).c_str());
    m.def("prepared_recurrent(Tensor qn, Tensor kn, Tensor v, Tensor gdecay, Tensor beta, Tensor(a!) out, "
          "Tensor(b!) state, Tensor indices, Tensor starts, Tensor? track_indices=None, "
          "Tensor? track_lens=None, bool track_state=False, int head_offset=0) -> ()");
    m.def("kda_varlen_recurrent_g(*, Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, "
          "Tensor(a!) initial_state_source, Tensor initial_state_indices, Tensor cu_seqlens, float scale, "
          "Tensor(b!)? intermediate_state=None, bool prefill=False, Tensor? track_state_indices=None, "
          "Tensor? track_state_lens=None) -> Tensor");
    m.def("kda_varlen_chunk_g(*, Tensor q, Tensor k, Tensor v, Tensor g, Tensor beta, "
          "Tensor(a!) initial_state_source, Tensor initial_state_indices, Tensor cu_seqlens, float scale, "
          "bool prefill=False, Tensor? track_state_indices=None, Tensor? track_state_lens=None) -> Tensor");
    m.def("move_intermediate_cache_kda(Tensor(a!) dst, Tensor src, Tensor dst_indices, Tensor src_indices, "
          "Tensor step_indices, int h_block_size=1) -> ()");
    m.def("kda_causal_conv1d(Tensor x, Tensor weight, Tensor? bias, Tensor(a!) conv_state, Tensor cache_indices, "
          "Tensor query_start_loc, Tensor? has_initial_state=None, Tensor? track_conv_indices=None, "
          "Tensor? track_conv_lens=None, int num_parts=3, bool silu=True) -> Tensor");
    m.def("kda_set_status_buffer(int device, Tensor? buf) -> ()");
    m.def("kda_abi_version() -> int");
    m.impl("kda_set_status_buffer", &kda_set_status_buffer);
    m.impl("kda_abi_version", &kda_abi_version_op);
}

TORCH_LIBRARY_IMPL(sgl_glm53_ascend, CUDA, m) {
    m.impl("kda_varlen_recurrent", &kda_varlen_recurrent);
    m.impl("kda_varlen_recurrent_v2", &kda_varlen_recurrent);
    m.impl("kda_varlen_chunk", &kda_varlen_chunk);
    m.impl("kda_varlen_chunk_v2", &kda_varlen_chunk);
    m.impl("prepared_recurrent", &prepared_recurrent);
    m.impl("kda_varlen_recurrent_g", &kda_varlen_recurrent_g);
    m.impl("kda_varlen_chunk_g", &kda_varlen_chunk_g);
    m.impl("move_intermediate_cache_kda", &move_intermediate_cache_kda);
    m.impl("kda_causal_conv1d", &kda_causal_conv1d);
}
