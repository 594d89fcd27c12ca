// Short causal convolution in front of the GLM KDA operator, on sm_100a,
// behind kda_conv_launch.
//
// The attention layer projects every token to one "mixed" row q | k | v
// (C channels), convolves each channel over the last W tokens of its own
// sequence (depthwise causal conv1d, W <= 4 taps, fp32 weights), applies SiLU
// and hands q, k and v to the KDA op. Each request keeps the last `window` raw
// input rows of its sequence in a bf16 conv-state pool slot, so a continued
// sequence (decode, a resumed prefix) sees the rows before its first new token.
// This is the step sglang's attention backend runs before the KDA op
// (AscendKDAAttnBackend.forward_extend, exercised by
// sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387).
//
// One pass over HBM, one launch, two kinds of CTA (each thread owns 8
// channels, one 16-byte bf16 vector, of a 1024-channel block):
//   * streaming CTAs, one per 16 tokens: load their rows (plus the W - 1
//     before them) first, look up their requests while the loads fly, and
//     write every output whose W rows lie inside its own request straight
//     into its plane of the [P][T][C/P] output (P = 3: q, k and v as the
//     contiguous tensors the KDA op reads). They never touch the conv state.
//   * request CTAs, one per request: the request's first W - 1 outputs (the
//     only ones that reach back into the old window), the tracked-prefix
//     checkpoint and the new window. Each loads every row it stores before its
//     first store, so the in-place window update needs no ordering between
//     CTAs: no other CTA reads the slot.

#include "kda_common.cuh"

namespace kda {
namespace conv {

constexpr int kThreads = 128;   // x 8 channels: 1024 channels per CTA
constexpr int kVec = 8;
constexpr int kTile = 16;       // tokens per streaming CTA
constexpr int kMaxWindow = 8;   // conv-state rows per slot (held in registers)
constexpr int kMeta = 32;       // requests a streaming CTA stages in shared memory

__device__ __forceinline__ void unpack8(const uint4 r, float *f) {
    f[0] = bf16_lo(r.x); f[1] = bf16_hi(r.x);
    f[2] = bf16_lo(r.y); f[3] = bf16_hi(r.y);
    f[4] = bf16_lo(r.z); f[5] = bf16_hi(r.z);
    f[6] = bf16_lo(r.w); f[7] = bf16_hi(r.w);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

__device__ __forceinline__ uint4 pack8(const float *f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}

__device__ __forceinline__ uint4 zero4() { return make_uint4(0u, 0u, 0u, 0u); }

// 1-, 4- or 8-byte per-request flag (torch bool, int32, int64).
__device__ __forceinline__ bool load_flag(const void *p, int bytes, int64_t i) {
    if (bytes == 1) return reinterpret_cast<const uint8_t *>(p)[i] != 0;
    return load_index(p, bytes, i) != 0;
}

struct Req {
    int64_t bos, eos, slot, tslot;
    int32_t code;   // 0, or the KDA_DEVICE_ERR_* that rejects the request
    bool init;      // reads the slot's rows before its first token
};

__device__ __forceinline__ Req load_req(const KdaConvArgs &p, int s) {
    Req q;
    q.bos = load_index(p.cu_seqlens, p.index_bytes[1], s);
    q.eos = load_index(p.cu_seqlens, p.index_bytes[1], s + 1);
    q.slot = load_index(p.indices, p.index_bytes[0], s);
    q.tslot = p.track_indices != nullptr ? load_index(p.track_indices, p.index_bytes[3], s) : 0;
    q.code = 0;
    if (q.bos < 0 || q.eos < q.bos || q.eos > p.num_tokens)
        q.code = KDA_DEVICE_ERR_BAD_SEQLENS;
    else if (q.slot < 0 || q.slot >= p.num_slots || q.tslot < 0 || q.tslot >= p.num_slots)
        q.code = KDA_DEVICE_ERR_BAD_SLOT;
    q.init = q.code == 0 && q.slot > 0 && (p.has_initial == nullptr || load_flag(p.has_initial, p.index_bytes[2], s));
    return q;
}

__device__ __forceinline__ uint4 *out_vec(const KdaConvArgs &p, int64_t t, int c) {
    const int cp = p.channels / p.num_parts;
    const int plane = c / cp;
    uint16_t *o = static_cast<uint16_t *>(p.out);
    return reinterpret_cast<uint4 *>(o + (static_cast<int64_t>(plane) * p.num_tokens + t) * cp + (c - plane * cp));
}

template <int W>
struct Taps {
    float w[W][kVec];
    float b[kVec];
};

template <int W>
__device__ __forceinline__ void load_taps(const KdaConvArgs &p, int c, Taps<W> &tp) {
    // weight [C][W]: this thread's 8 channels are 8 * W consecutive floats.
    const float *wp = p.weight + static_cast<int64_t>(c) * W;
#pragma unroll
    for (int j = 0; j < kVec; ++j)
#pragma unroll
        for (int k = 0; k < W; ++k) tp.w[k][j] = __ldg(wp + j * W + k);
#pragma unroll
    for (int j = 0; j < kVec; ++j) tp.b[j] = p.bias != nullptr ? __ldg(p.bias + c + j) : 0.0f;
}

// SiLU on the fp32 accumulator. The output is rounded to bf16 (8-bit
// mantissa), so the fast exponential and division (relative errors of a few
// 2^-22) change a result only where it sits on a bf16 rounding boundary.
__device__ __forceinline__ float silu(float a) {
    return __fdividef(a, 1.0f + __expf(fminf(-a, 80.0f)));
}

// out = act(bias + sum_k w[k] * row_k), taps in order k = 0..W-1 over the W
// rows oldest first (row W-1 is the token itself); one rounding to bf16.
template <int W>
__device__ __forceinline__ uint4 conv_out(const KdaConvArgs &p, const Taps<W> &tp, const float (*win)[kVec]) {
    float y[kVec];
#pragma unroll
    for (int j = 0; j < kVec; ++j) {
        float acc = tp.b[j];
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(tp.w[k][j], win[k][j], acc);
        y[j] = p.activation == KDA_CONV_ACT_SILU ? silu(acc) : acc;
    }
    return pack8(y);
}

// The number of requests r in [0, R) whose entry cu_seqlens[r + off] is
// <= bound (inclusive) or < bound (strict): for a monotone cu_seqlens, the
// first request index past that bound. A warp-wide 32-ary search, called by
// all 32 lanes of one warp; on a non-monotone array it still ends, with a
// value in [0, R].
__device__ __forceinline__ int count_below(const KdaConvArgs &p, int off, int64_t bound, bool inclusive) {
    const int lane = threadIdx.x & 31;
    int lo = 0, hi = p.num_req;
    while (lo < hi) {
        const int n = hi - lo;
        const int stride = (n + 31) / 32;
        const int pos = lo + (lane + 1) * stride - 1;
        bool pred = false;
        if (pos < hi) {
            const int64_t v = load_index(p.cu_seqlens, p.index_bytes[1], pos + off);
            pred = inclusive ? v <= bound : v < bound;
        }
        const int tested = n / stride;
        const int k = __popc(__ballot_sync(0xffffffffu, pred));
        const int new_lo = lo + k * stride;
        hi = k < tested ? new_lo + stride - 1 : hi;
        lo = new_lo < hi ? new_lo : hi;
    }
    return lo;
}

// ---------------------------------------------------------------------------
// Request CTAs: one request x 1024 channels, the only threads that touch the
// conv state. Per thread (8 channels): the old window (when the request
// continues), the request's first min(len, W-1) outputs (the ones whose rows
// reach back before its first token), the tracked-prefix checkpoint and the
// new window. Every row a store needs is loaded before the first store, so
// the in-place window update reads the old values.
// ---------------------------------------------------------------------------

template <int W>
__device__ __forceinline__ void request_block(const KdaConvArgs &p, int r, int c) {
    const Req q = load_req(p, r);
    if (q.code != 0) {
        if (c == 0) report(p.status, q.code);
        if (q.code == KDA_DEVICE_ERR_BAD_SEQLENS) return;
        for (int64_t t = q.bos; t < q.eos && t < q.bos + (W - 1); ++t) *out_vec(p, t, c) = zero4();
        return;
    }
    const uint16_t *x = static_cast<const uint16_t *>(p.x);
    uint16_t *st = static_cast<uint16_t *>(p.conv_state);
    const int64_t len = q.eos - q.bos;
    const int win = p.window;
    // Old window, oldest row first (zeros for a fresh request or the padding slot).
    uint4 old[kMaxWindow];
#pragma unroll
    for (int j = 0; j < kMaxWindow; ++j)
        old[j] = (q.init && j < win)
                     ? *reinterpret_cast<const uint4 *>(st + q.slot * p.state_stride[0] + j * p.state_stride[1] + c)
                     : zero4();
    // The request's first W-1 token rows.
    uint4 head[W > 1 ? W - 1 : 1];
#pragma unroll
    for (int i = 0; i < W - 1; ++i)
        head[i] = i < len ? __ldg(reinterpret_cast<const uint4 *>(x + (q.bos + i) * p.x_row_stride + c)) : zero4();
    Taps<W> tp;
    load_taps<W>(p, c, tp);
    // History row rr of the request: rr < 0 the old window's row win + rr,
    // 0 <= rr < W - 1 a head row (selected from registers, no local memory).
    auto early = [&](int rr) -> uint4 {
        uint4 v = zero4();
#pragma unroll
        for (int j = 0; j < kMaxWindow; ++j)
            if (rr == j - win) v = old[j];
#pragma unroll
        for (int i = 0; i < W - 1; ++i)
            if (rr == i) v = head[i];
        return v;
    };
#pragma unroll
    for (int i = 0; i < W - 1; ++i) {
        if (i < len) {
            float w[W][kVec];
#pragma unroll
            for (int k = 0; k < W; ++k) unpack8(early(i - (W - 1) + k), w[k]);
            *out_vec(p, q.bos + i, c) = conv_out<W>(p, tp, w);
        }
    }
    // Checkpoint and new window: history rows tl - win .. tl - 1 for tl = the
    // tracked length and tl = len.
    auto row_at = [&](int64_t rr) -> uint4 {
        if (rr >= 0) return __ldg(reinterpret_cast<const uint4 *>(x + (q.bos + rr) * p.x_row_stride + c));
        return early(static_cast<int>(rr));
    };
    if (q.tslot > 0) {
        const int64_t tlen = load_index(p.track_lens, p.index_bytes[4], r);
        if (tlen >= 0 && tlen <= len) {
            uint4 rows[kMaxWindow];
#pragma unroll
            for (int j = 0; j < kMaxWindow; ++j) rows[j] = j < win ? row_at(tlen - win + j) : zero4();
#pragma unroll
            for (int j = 0; j < kMaxWindow; ++j)
                if (j < win)
                    *reinterpret_cast<uint4 *>(st + q.tslot * p.state_stride[0] + j * p.state_stride[1] + c) = rows[j];
        }
    }
    if (q.slot > 0 && len > 0) {
        uint4 rows[kMaxWindow];
#pragma unroll
        for (int j = 0; j < kMaxWindow; ++j) rows[j] = j < win ? row_at(len - win + j) : zero4();
#pragma unroll
        for (int j = 0; j < kMaxWindow; ++j)
            if (j < win)
                *reinterpret_cast<uint4 *>(st + q.slot * p.state_stride[0] + j * p.state_stride[1] + c) = rows[j];
    }
}

// ---------------------------------------------------------------------------
// Streaming CTAs: kTile tokens x 1024 channels. Every output whose W rows lie
// inside its own request (t >= bos + W - 1), from token rows only; zeros for
// tokens no request covers and for rejected requests. The rows are loaded
// before the CTA looks up its requests, so the lookup hides under them.
// ---------------------------------------------------------------------------

struct TileMeta {
    int64_t bos[kMeta];
    int64_t eos[kMeta];
    int32_t bad[kMeta];
    int first;   // request index of entry 0
    int count;   // valid entries
};

template <int W>
__device__ __forceinline__ void stream_block(const KdaConvArgs &p, int64_t t0, int c, TileMeta &m) {
    constexpr int kRows = kTile + W - 1;
    const uint16_t *x = static_cast<const uint16_t *>(p.x);
    const bool active = c < p.channels;
    uint4 rows[kRows];   // rows[i] = token t0 - (W - 1) + i
#pragma unroll
    for (int i = 0; i < kRows; ++i) {
        const int64_t t = t0 - (W - 1) + i;
        rows[i] = (active && t >= 0 && t < p.num_tokens)
                      ? __ldg(reinterpret_cast<const uint4 *>(x + t * p.x_row_stride + c))
                      : zero4();
    }
    if (threadIdx.x < 32) {
        const int f = count_below(p, 1, t0, true);   // first request ending after t0
        const int lane = threadIdx.x;
        if (f + lane < p.num_req) {
            const Req q = load_req(p, f + lane);
            m.bos[lane] = q.bos;
            m.eos[lane] = q.eos;
            m.bad[lane] = q.code;
        }
        if (lane == 0) {
            m.first = f;
            m.count = min(kMeta, p.num_req - f);
        }
    }
    __syncthreads();
    if (!active) return;
    Taps<W> tp;
    load_taps<W>(p, c, tp);
    float win[W][kVec];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) unpack8(rows[k], win[k]);
    int e = 0;
    int64_t bos = -1, eos = -1;
    int32_t bad = 1;
#pragma unroll
    for (int i = 0; i < kTile; ++i) {
        const int64_t t = t0 + i;
        unpack8(rows[i + W - 1], win[W - 1]);
        if (t < p.num_tokens) {
            if (t >= eos) {
                // the request holding t: staged entries first, then global loads
                while (e < m.count && m.eos[e] <= t) ++e;
                if (e < m.count) {
                    bos = m.bos[e];
                    eos = m.eos[e];
                    bad = m.bad[e];
                } else {
                    int s = m.first + e;
                    while (s < p.num_req && load_index(p.cu_seqlens, p.index_bytes[1], s + 1) <= t) ++s;
                    if (s < p.num_req) {
                        const Req q = load_req(p, s);
                        bos = q.bos;
                        eos = q.eos;
                        bad = q.code;
                    } else {
                        bos = eos = p.num_tokens + 1;
                        bad = KDA_DEVICE_ERR_BAD_SEQLENS;
                    }
                }
            }
            if (t < bos || bad == KDA_DEVICE_ERR_BAD_SEQLENS) {
                *out_vec(p, t, c) = zero4();   // no (valid) request covers t
            } else if (t >= bos + (W - 1)) {
                // the request CTA writes the first W - 1 rows, zeros included
                *out_vec(p, t, c) = bad != 0 ? zero4() : conv_out<W>(p, tp, win);
            }
        }
#pragma unroll
        for (int k = 0; k + 1 < W; ++k)
#pragma unroll
            for (int j = 0; j < kVec; ++j) win[k][j] = win[k + 1][j];
    }
}

template <int W>
__global__ void __launch_bounds__(kThreads) conv_kernel(const KdaConvArgs p, int num_stream_blocks) {
    __shared__ TileMeta meta;
    const int c = (blockIdx.y * kThreads + threadIdx.x) * kVec;
    if (static_cast<int>(blockIdx.x) < num_stream_blocks) {
        stream_block<W>(p, static_cast<int64_t>(blockIdx.x) * kTile, c, meta);
    } else if (c < p.channels) {
        request_block<W>(p, static_cast<int>(blockIdx.x) - num_stream_blocks, c);
    }
}

template <int W>
cudaError_t launch_w(const KdaConvArgs &a, cudaStream_t st) {
    const int64_t tiles = (static_cast<int64_t>(a.num_tokens) + kTile - 1) / kTile;
    const dim3 grid(static_cast<unsigned>(tiles + a.num_req),
                    static_cast<unsigned>((a.channels + kThreads * kVec - 1) / (kThreads * kVec)));
    conv_kernel<W><<<grid, kThreads, 0, st>>>(a, static_cast<int>(tiles));
    return cudaGetLastError();
}

}  // namespace conv
}  // namespace kda

extern "C" int kda_conv_launch(const KdaConvArgs *args, void *stream) {
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    const KdaConvArgs &a = *args;
    if (a.num_req < 0 || a.num_tokens < 0 || a.channels <= 0 || a.num_parts <= 0 || a.num_slots < 0)
        return KDA_ERR_INVALID_ARGUMENT;
    if (a.width < 1 || a.width > 4) return KDA_ERR_UNSUPPORTED;
    if (a.window < a.width - 1 || a.window < 0) return KDA_ERR_INVALID_ARGUMENT;
    if (a.window > kda::conv::kMaxWindow) return KDA_ERR_UNSUPPORTED;
    if (a.activation != KDA_CONV_ACT_NONE && a.activation != KDA_CONV_ACT_SILU) return KDA_ERR_UNSUPPORTED;
    if (a.index_bytes[0] != 4 && a.index_bytes[0] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (a.index_bytes[1] != 4 && a.index_bytes[1] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (a.has_initial != nullptr && a.index_bytes[2] != 1 && a.index_bytes[2] != 4 && a.index_bytes[2] != 8)
        return KDA_ERR_INVALID_ARGUMENT;
    if ((a.track_indices == nullptr) != (a.track_lens == nullptr)) return KDA_ERR_INVALID_ARGUMENT;
    if (a.track_indices != nullptr &&
        ((a.index_bytes[3] != 4 && a.index_bytes[3] != 8) || (a.index_bytes[4] != 4 && a.index_bytes[4] != 8)))
        return KDA_ERR_INVALID_ARGUMENT;
    if (a.num_req == 0 && a.num_tokens == 0) return KDA_OK;
    if (a.channels % a.num_parts != 0) return KDA_ERR_INVALID_ARGUMENT;
    // With no requests the launch only zeroes the output (no metadata is read).
    if (a.weight == nullptr || (a.num_req > 0 && (a.indices == nullptr || a.cu_seqlens == nullptr)) ||
        (a.num_tokens > 0 && (a.x == nullptr || a.out == nullptr)) || (a.window > 0 && a.conv_state == nullptr))
        return KDA_ERR_INVALID_ARGUMENT;
    if (a.x_row_stride < a.channels) return KDA_ERR_INVALID_ARGUMENT;
    // 16-byte vectors: 8 channels never straddle an output plane or a row.
    const int64_t cp = a.channels / a.num_parts;
    if (a.channels % 8 != 0 || cp % 8 != 0 || a.x_row_stride % 8 != 0 || a.state_stride[0] % 8 != 0 ||
        a.state_stride[1] % 8 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.conv_state) & 15u) != 0)
        return KDA_ERR_ALIGNMENT;
    if ((static_cast<int64_t>(a.num_tokens) + kda::conv::kTile - 1) / kda::conv::kTile + a.num_req > 0x7fffffff)
        return KDA_ERR_TOO_LARGE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    switch (a.width) {
        case 1: e = kda::conv::launch_w<1>(a, st); break;
        case 2: e = kda::conv::launch_w<2>(a, st); break;
        case 3: e = kda::conv::launch_w<3>(a, st); break;
        default: e = kda::conv::launch_w<4>(a, st); break;
    }
    return e == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
