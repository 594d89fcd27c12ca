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
// One pass over HBM in two kernels on the stream:
//   * the request kernel, one CTA per (request, 1024 channels; 8 channels per
//     thread): the request's first W - 1 outputs (the only ones that reach
//     back into the old window), the tracked-prefix checkpoint and the new
//     window. It loads every row it stores before its first store, so the
//     in-place window update needs no ordering between CTAs: no other CTA
//     reads the slot. In batches of short requests (decode, verify: at most 4
//     tokens per request on average) it computes every token, zeroes the rows
//     no request covers, and is the only launch.
//   * the streaming kernel, one CTA per (64 tokens, 1024 channels; 8 channels
//     per thread): every other output, from token rows only, straight into its
//     plane of the [P][T][C/P] output (P = 3: q, k and v as the contiguous
//     tensors the KDA op reads), with the next 4 rows loading while the
//     current 4 compute. It never touches the conv state, so the two kernels
//     need no ordering either; it also zeroes the rows no request covers.

#include "kda_common.cuh"

#include <climits>

namespace kda {
namespace conv {

constexpr int kThreads = 128;
constexpr int kReqVec = 8;      // channels per thread in the request kernel (1024 per CTA)
constexpr int kStreamVec = 8;   // channels per thread in the streaming kernel (1024 per CTA)
constexpr int kSpan = 64;       // tokens per streaming CTA
constexpr int kSub = 4;         // tokens per sub-tile (rows in flight per thread)
constexpr int kMaxWindow = 8;   // conv-state rows per slot
constexpr int kReqSub = 4;      // token rows the request kernel loads per batch
constexpr int kMeta = 64;       // requests a streaming CTA stages in shared memory
constexpr int kShortAvg = 4;    // tokens per request at or below which the request kernel takes every token

// V bf16 channels as one vector: 16 bytes (V = 8) or 8 bytes (V = 4).
template <int V> struct Vec;
template <> struct Vec<8> { using T = uint4; };
template <> struct Vec<4> { using T = uint2; };

__device__ __forceinline__ void unpack(const uint4 r, float *f) {
    f[0] = bf16_lo(r.x); f[1] = bf16_hi(r.x);
    f[2] = bf16_lo(r.y); f[3] = bf16_hi(r.y);
    f[4] = bf16_lo(r.z); f[5] = bf16_hi(r.z);
    f[6] = bf16_lo(r.w); f[7] = bf16_hi(r.w);
}

__device__ __forceinline__ void unpack(const uint2 r, float *f) {
    f[0] = bf16_lo(r.x); f[1] = bf16_hi(r.x);
    f[2] = bf16_lo(r.y); f[3] = bf16_hi(r.y);
}

__device__ __forceinline__ uint32_t pack2(float a, float b) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

template <int V>
__device__ __forceinline__ typename Vec<V>::T pack(const float *f);
template <>
__device__ __forceinline__ uint4 pack<8>(const float *f) {
    return make_uint4(pack2(f[0], f[1]), pack2(f[2], f[3]), pack2(f[4], f[5]), pack2(f[6], f[7]));
}
template <>
__device__ __forceinline__ uint2 pack<4>(const float *f) {
    return make_uint2(pack2(f[0], f[1]), pack2(f[2], f[3]));
}

template <int V>
__device__ __forceinline__ typename Vec<V>::T zero() {
    typename Vec<V>::T z;
    uint32_t *w = reinterpret_cast<uint32_t *>(&z);
#pragma unroll
    for (int i = 0; i < V / 2; ++i) w[i] = 0u;
    return z;
}

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

// Request metadata; every load is independent of the others (one round trip).
__device__ __forceinline__ Req load_req(const KdaConvArgs &p, int s) {
    Req q;
    q.bos = load_index(p.cu_seqlens, p.index_bytes[1], s);
    q.eos = load_index(p.cu_seqlens, p.index_bytes[1], s + 1);
    q.slot = load_index(p.indices, p.index_bytes[0], s);
    q.tslot = p.track_indices != nullptr ? load_index(p.track_indices, p.index_bytes[3], s) : 0;
    const bool cont = p.has_initial == nullptr || load_flag(p.has_initial, p.index_bytes[2], s);
    q.code = 0;
    if (q.bos < 0 || q.eos < q.bos || q.eos > p.num_tokens)
        q.code = KDA_DEVICE_ERR_BAD_SEQLENS;
    else if (q.slot < 0 || q.slot >= p.num_slots || q.tslot < 0 || q.tslot >= p.num_slots)
        q.code = KDA_DEVICE_ERR_BAD_SLOT;
    q.init = q.code == 0 && q.slot > 0 && cont;
    return q;
}

// This thread's column of the output: token t's V channels are at
// base + t * stride (one plane of [P][T][C/P]); computed once per thread.
template <int V>
struct OutCol {
    uint16_t *base;
    int64_t stride;
    __device__ __forceinline__ typename Vec<V>::T *at(int64_t t) const {
        return reinterpret_cast<typename Vec<V>::T *>(base + t * stride);
    }
};

template <int V>
__device__ __forceinline__ OutCol<V> out_col(const KdaConvArgs &p, int c) {
    const int cp = p.channels / p.num_parts;
    const int plane = c / cp;
    OutCol<V> o;
    o.base = static_cast<uint16_t *>(p.out) + static_cast<int64_t>(plane) * p.num_tokens * cp + (c - plane * cp);
    o.stride = cp;
    return o;
}

template <int W, int V>
struct Taps {
    float w[W][V];
    float b[V];
};

template <int W, int V>
__device__ __forceinline__ void load_taps(const KdaConvArgs &p, int c, Taps<W, V> &tp) {
    // weight [C][W]: this thread's V channels are V * W consecutive floats,
    // 16-byte aligned (c is a multiple of V, the arrays 16-byte aligned).
    const float4 *wp = reinterpret_cast<const float4 *>(p.weight + static_cast<int64_t>(c) * W);
    float f[V * W];
#pragma unroll
    for (int v = 0; v < V * W / 4; ++v) {
        const float4 q = __ldg(wp + v);
        f[4 * v] = q.x; f[4 * v + 1] = q.y; f[4 * v + 2] = q.z; f[4 * v + 3] = q.w;
    }
#pragma unroll
    for (int j = 0; j < V; ++j)
#pragma unroll
        for (int k = 0; k < W; ++k) tp.w[k][j] = f[j * W + k];
    if (p.bias != nullptr) {
#pragma unroll
        for (int v = 0; v < V / 4; ++v) {
            const float4 b = __ldg(reinterpret_cast<const float4 *>(p.bias + c) + v);
            tp.b[4 * v] = b.x; tp.b[4 * v + 1] = b.y; tp.b[4 * v + 2] = b.z; tp.b[4 * v + 3] = b.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < V; ++j) tp.b[j] = 0.0f;
    }
}

// SiLU on the fp32 accumulator: a * 1 / (1 + 2^(-a log2 e)) with the
// hardware's approximate base-2 exponential and reciprocal (PTX ex2.approx,
// rcp.approx; relative errors around 2^-22). The output is rounded to bf16
// (8-bit mantissa), so they change a result only where it sits on a bf16
// rounding boundary. For a very negative a the exponential overflows to +inf
// and the reciprocal gives 0: the result is -0, as the bf16 rounding of the
// true value (below 1e-40) would be.
__device__ __forceinline__ float silu(float a) {
    constexpr float kLog2e = 1.4426950408889634f;
    float e, r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-a * kLog2e));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(1.0f + e));
    return a * r;
}

// out = act(bias + sum_k w[k] * row_k), taps in order k = 0..W-1 over the W
// rows oldest first (row W-1 is the token itself); one rounding to bf16.
template <int W, int V>
__device__ __forceinline__ typename Vec<V>::T conv_out(const KdaConvArgs &p, const Taps<W, V> &tp,
                                                      const float (*win)[V]) {
    float y[V];
#pragma unroll
    for (int j = 0; j < V; ++j) {
        float acc = tp.b[j];
#pragma unroll
        for (int k = 0; k < W; ++k) acc = fmaf(tp.w[k][j], win[k][j], acc);
        y[j] = p.activation == KDA_CONV_ACT_SILU ? silu(acc) : acc;
    }
    return pack<V>(y);
}

template <int W, int V>
__device__ __forceinline__ void shift_window(float (*win)[V]) {
#pragma unroll
    for (int k = 0; k + 1 < W; ++k)
#pragma unroll
        for (int j = 0; j < V; ++j) win[k][j] = win[k + 1][j];
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
// Request kernel: one CTA per (request, 1024 channels), the only threads that
// touch the conv state. Per thread (8 channels): the request's first `head`
// outputs (W - 1, the ones whose rows reach back before its first token; or
// all of them for batches of short requests), then the tracked-prefix
// checkpoint and the new window. Every row the state stores need is loaded
// (from the tokens or the old window in memory) before the first store, so the
// in-place window update reads the old values.
// ---------------------------------------------------------------------------

template <int W, int MAXWIN>
__global__ void __launch_bounds__(kThreads, 5) conv_request_kernel(const KdaConvArgs p, int head) {
    constexpr int V = kReqVec;
    using VT = typename Vec<V>::T;
    const int c = (blockIdx.y * kThreads + threadIdx.x) * V;
    if (c >= p.channels) return;
    const int r = blockIdx.x;
    Taps<W, V> tp;
    load_taps<W, V>(p, c, tp);          // independent of the request: overlaps its metadata
    const Req q = load_req(p, r);
    const OutCol<V> oc = out_col<V>(p, c);
    const int64_t len = q.eos - q.bos;
    const int64_t n_out = len < head ? len : head;
    if (head == INT_MAX && q.code != KDA_DEVICE_ERR_BAD_SEQLENS) {
        // Short batch, one launch: the first and the last request also zero the
        // rows no request covers (before the first and after the last request;
        // 0 <= bos <= eos <= T here).
        if (r == 0)
            for (int64_t t = 0; t < q.bos; ++t) *oc.at(t) = zero<V>();
        if (r == p.num_req - 1)
            for (int64_t t = q.eos; t < p.num_tokens; ++t) *oc.at(t) = zero<V>();
    }
    if (q.code != 0) {
        if (c == 0) report(p.status, q.code);
        if (q.code == KDA_DEVICE_ERR_BAD_SEQLENS) return;
        for (int64_t t = 0; t < n_out; ++t) *oc.at(q.bos + t) = zero<V>();
        return;
    }
    const uint16_t *x = static_cast<const uint16_t *>(p.x);
    uint16_t *st = static_cast<uint16_t *>(p.conv_state);
    const int win = p.window;
    // History row rr of the request (rr < 0: row win + rr of the old window,
    // zeros for a fresh request; rr >= 0: its token rows). Plain loads for
    // the state: this thread stores to it later.
    auto row_at = [&](int64_t rr) -> VT {
        if (rr >= 0) return __ldg(reinterpret_cast<const VT *>(x + (q.bos + rr) * p.x_row_stride + c));
        if (!q.init) return zero<V>();
        return *reinterpret_cast<const VT *>(st + q.slot * p.state_stride[0] + (win + rr) * p.state_stride[1] + c);
    };
    float w[W][V];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) unpack(row_at(k - (W - 1)), w[k]);
    for (int64_t i0 = 0; i0 < n_out; i0 += kReqSub) {
        VT rows[kReqSub];
#pragma unroll
        for (int i = 0; i < kReqSub; ++i) rows[i] = i0 + i < n_out ? row_at(i0 + i) : zero<V>();
#pragma unroll
        for (int i = 0; i < kReqSub; ++i) {
            if (i0 + i < n_out) {
                unpack(rows[i], w[W - 1]);
                *oc.at(q.bos + i0 + i) = conv_out<W, V>(p, tp, w);
            }
            shift_window<W, V>(w);
        }
    }
    // Checkpoint rows tl - win .. tl - 1 (tl = the tracked length) and new
    // window rows len - win .. len - 1, all loaded before any state store.
    int64_t tlen = -1;
    if (q.tslot > 0) tlen = load_index(p.track_lens, p.index_bytes[4], r);
    const bool ckpt = q.tslot > 0 && tlen >= 0 && tlen <= len;
    const bool upd = q.slot > 0 && len > 0;
    VT ck[MAXWIN], nw[MAXWIN];
#pragma unroll
    for (int j = 0; j < MAXWIN; ++j) {
        ck[j] = (ckpt && j < win) ? row_at(tlen - win + j) : zero<V>();
        nw[j] = (upd && j < win) ? row_at(len - win + j) : zero<V>();
    }
#pragma unroll
    for (int j = 0; j < MAXWIN; ++j) {
        if (ckpt && j < win)
            *reinterpret_cast<VT *>(st + q.tslot * p.state_stride[0] + j * p.state_stride[1] + c) = ck[j];
        if (upd && j < win)
            *reinterpret_cast<VT *>(st + q.slot * p.state_stride[0] + j * p.state_stride[1] + c) = nw[j];
    }
}

// ---------------------------------------------------------------------------
// Streaming kernel: one CTA per (kSpan tokens, 1024 channels). Every output of
// a request past its first `head` tokens, from token rows only; zeros for
// tokens no request covers and for rejected requests. The span is walked in
// sub-tiles of kSub tokens, the next sub-tile's rows loading while the
// current one computes; the CTA's first rows are issued before it looks up
// its requests, so the lookup hides under them. With ZERO_ONLY (a batch with
// no requests) it only zeroes the rows.
// ---------------------------------------------------------------------------

struct TileMeta {
    int64_t bos[kMeta];
    int64_t eos[kMeta];
    int32_t bad[kMeta];
    int first;   // request index of entry 0
    int count;   // valid entries
};

// The request holding token t (t >= the current eos): the staged entries
// first, then global loads past them.
__device__ __forceinline__ void find_request(const KdaConvArgs &p, const TileMeta &m, int64_t t, int &e,
                                             int64_t &bos, int64_t &eos, int32_t &bad) {
    while (e < m.count && m.eos[e] <= t) ++e;
    if (e < m.count) {
        bos = m.bos[e];
        eos = m.eos[e];
        bad = m.bad[e];
        return;
    }
    int sq = m.first + e;
    while (sq < p.num_req && load_index(p.cu_seqlens, p.index_bytes[1], sq + 1) <= t) ++sq;
    if (sq < p.num_req) {
        const Req q = load_req(p, sq);
        bos = q.bos;
        eos = q.eos;
        bad = q.code;
    } else {
        bos = eos = p.num_tokens + 1;
        bad = KDA_DEVICE_ERR_BAD_SEQLENS;
    }
}

template <int W, bool ZERO_ONLY>
__global__ void __launch_bounds__(kThreads, 4) conv_stream_kernel(const KdaConvArgs p) {
    constexpr int V = kStreamVec;
    using VT = typename Vec<V>::T;
    constexpr int kH = W > 1 ? W - 1 : 1;
    __shared__ TileMeta m;
    const int64_t t0 = static_cast<int64_t>(blockIdx.x) * kSpan;
    const int c = (blockIdx.y * kThreads + threadIdx.x) * V;
    const bool active = c < p.channels;
    const uint16_t *x = static_cast<const uint16_t *>(p.x);
    auto load_row = [&](int64_t t) -> VT {
        return (!ZERO_ONLY && active && t >= 0 && t < p.num_tokens)
                   ? __ldg(reinterpret_cast<const VT *>(x + t * p.x_row_stride + c))
                   : zero<V>();
    };
    VT halo[kH], nxt[kSub];
#pragma unroll
    for (int k = 0; k < W - 1; ++k) halo[k] = load_row(t0 - (W - 1) + k);
#pragma unroll
    for (int i = 0; i < kSub; ++i) nxt[i] = load_row(t0 + i);
    if (threadIdx.x < 64) {
        // warps 0 and 1 each find the first request ending after t0 and
        // stage 32 requests from there on
        const int f = count_below(p, 1, t0, true);
        const int e = threadIdx.x;
        if (f + e < p.num_req) {
            const Req q = load_req(p, f + e);
            m.bos[e] = q.bos;
            m.eos[e] = q.eos;
            m.bad[e] = q.code;
        }
        if (e == 0) {
            m.first = f;
            m.count = min(kMeta, p.num_req - f);
        }
    }
    __syncthreads();
    if (!active) return;
    const OutCol<V> oc = out_col<V>(p, c);
    int e = 0;
    int64_t bos = -1, eos = -1;
    int32_t bad = 1;
    if constexpr (ZERO_ONLY) {
        for (int i = 0; i < kSpan; ++i) {
            const int64_t t = t0 + i;
            if (t >= p.num_tokens) break;
            if (t >= eos) find_request(p, m, t, e, bos, eos, bad);
            if (t < bos || bad == KDA_DEVICE_ERR_BAD_SEQLENS) *oc.at(t) = zero<V>();
        }
        return;
    } else {
        Taps<W, V> tp;
        load_taps<W, V>(p, c, tp);
        float win[W][V];
#pragma unroll
        for (int k = 0; k < W - 1; ++k) unpack(halo[k], win[k]);
#pragma unroll 1
        for (int s = 0; s < kSpan / kSub; ++s) {
            VT cur[kSub];
#pragma unroll
            for (int i = 0; i < kSub; ++i) cur[i] = nxt[i];
            const int64_t ts = t0 + s * kSub;
            if (ts >= p.num_tokens) break;
            if (s + 1 < kSpan / kSub) {
#pragma unroll
                for (int i = 0; i < kSub; ++i) nxt[i] = load_row(ts + kSub + i);
            }
            if (ts >= eos) find_request(p, m, ts, e, bos, eos, bad);
            if (bad == 0 && ts >= bos + (W - 1) && ts + kSub <= eos) {
                // the whole sub-tile inside one request, past its first W - 1 tokens
#pragma unroll
                for (int i = 0; i < kSub; ++i) {
                    unpack(cur[i], win[W - 1]);
                    *oc.at(ts + i) = conv_out<W, V>(p, tp, win);
                    shift_window<W, V>(win);
                }
                continue;
            }
#pragma unroll
            for (int i = 0; i < kSub; ++i) {
                const int64_t t = ts + i;
                unpack(cur[i], win[W - 1]);
                if (t < p.num_tokens) {
                    if (t >= eos) find_request(p, m, t, e, bos, eos, bad);
                    if (t < bos || bad == KDA_DEVICE_ERR_BAD_SEQLENS) {
                        *oc.at(t) = zero<V>();   // no (valid) request covers t
                    } else if (t >= bos + (W - 1)) {
                        // the request kernel writes the first W - 1 rows, zeros included
                        *oc.at(t) = bad != 0 ? zero<V>() : conv_out<W, V>(p, tp, win);
                    }
                }
                shift_window<W, V>(win);
            }
        }
    }
}

template <int W>
cudaError_t launch_w(const KdaConvArgs &a, cudaStream_t st) {
    // Batches of short requests (decode, verify): the request kernel computes
    // every token and zeroes the uncovered rows; no second launch.
    const bool short_batch = a.num_req > 0 && a.num_tokens <= static_cast<int64_t>(kShortAvg) * a.num_req;
    if (a.num_req > 0) {
        const dim3 grid(a.num_req, (a.channels + kThreads * kReqVec - 1) / (kThreads * kReqVec));
        const int head = short_batch ? INT_MAX : W - 1;
        if (a.window <= 4)
            conv_request_kernel<W, 4><<<grid, kThreads, 0, st>>>(a, head);
        else
            conv_request_kernel<W, kMaxWindow><<<grid, kThreads, 0, st>>>(a, head);
    }
    const int64_t spans = (static_cast<int64_t>(a.num_tokens) + kSpan - 1) / kSpan;
    if (spans > 0 && !short_batch) {
        const dim3 grid(static_cast<unsigned>(spans), (a.channels + kThreads * kStreamVec - 1) / (kThreads * kStreamVec));
        if (a.num_req == 0)
            conv_stream_kernel<W, true><<<grid, kThreads, 0, st>>>(a);
        else
            conv_stream_kernel<W, false><<<grid, kThreads, 0, st>>>(a);
    }
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
    // 8- and 16-byte vectors: a thread's channels never straddle an output
    // plane or a row.
    const int64_t cp = a.channels / a.num_parts;
    if (a.channels % 8 != 0 || cp % 8 != 0 || a.x_row_stride % 8 != 0 || a.state_stride[0] % 8 != 0 ||
        a.state_stride[1] % 8 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(a.out) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.conv_state) & 15u) != 0 ||
        (reinterpret_cast<uintptr_t>(a.weight) & 15u) != 0 || (reinterpret_cast<uintptr_t>(a.bias) & 15u) != 0)
        return KDA_ERR_ALIGNMENT;
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
