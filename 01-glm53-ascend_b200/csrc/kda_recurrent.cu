// Token-at-a-time GLM KDA recurrence on sm_100a: decode, verify (per-step
// checkpoints) and recurrent prefill, behind kda_recurrent_launch and
// kda_prepared_recurrent_launch.
//
// Math per token t, head h (kda_python.py:271-303; decode kernel
// sgl-glm53-ascend-ops/csrc/kda/recurrent/kda_varlen_recurrent_decode.h:630-741):
//   S <- Diag(e^g) S ; pred = S^T kn ; delta = beta (v - pred) ;
//   S <- S + kn delta^T ; o = S^T qn
// The pool slot is physically [V][K] (K contiguous), so a value row of the
// state is D contiguous floats and every row is independent given kn, qn,
// e^g and beta.
//
// Work decomposition (B200-first, no counterpart in the reference):
//   * one CTA per (request, head, 32-row value slice): 128 threads, 4 warps,
//     8 value rows per warp, 8 lanes per row, each lane D/8 key elements in
//     float4 groups (k = c*32 + sub*4 + e), so every global or shared access
//     of a row is 128 contiguous bytes per 8 lanes.
//   * the 32 x D fp32 slice (16 KiB at D=128) is staged into shared memory by
//     one bulk TMA copy (cp.async.bulk, no multicast) while the warps compute
//     the token prologue; the state then lives in registers for all tokens of
//     the request.
//   * the prologue (L2 norms, gate, beta) is computed per warp with
//     8-lane shuffles; row reductions are 3 xor-shuffles per row quad.
//   * write-back, per-step checkpoints and prefix checkpoints are coalesced
//     float4 stores straight from registers.
// The kernel is HBM-bound: 2 x 64 KiB of state traffic per (token, head) in
// decode against ~1.5 KB of token inputs.

#include "kda_common.cuh"

namespace kda {

constexpr int kBV = 32;            // value rows per CTA
constexpr int kRowsPerWarp = 8;
constexpr int kRecThreads = kBV / kRowsPerWarp * 32;  // 128

template <int D, int MODE>
struct TokenRaw {
    static constexpr int NC = D / 32;
    uint2 qb[NC], kb[NC];      // bf16 q, k (RAW, LOG)
    float4 qf[NC], kf[NC];     // fp32 qn, kn (PREPARED)
    float4 gf[NC];             // log-decay (LOG) or exp(g) (PREPARED)
    uint2 ab[NC];              // bf16 a (RAW)
    uint16_t vb[2];            // this lane's two value rows
    float beta;                // LOG / PREPARED
    uint16_t bb;               // RAW
};

template <int D, int MODE>
__device__ __forceinline__ void load_token(TokenRaw<D, MODE> &r, const KdaArgs &p, int64_t t, int h,
                                           int sub, int row0) {
    constexpr int NC = D / 32;
    const int64_t base = (t * p.num_heads + h) * D;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int64_t off = base + c * 32 + sub * 4;
        if constexpr (MODE == KDA_GATE_PREPARED) {
            r.qf[c] = load_f32x4(static_cast<const float *>(p.q), off);
            r.kf[c] = load_f32x4(static_cast<const float *>(p.k), off);
            r.gf[c] = load_f32x4(p.g, off);
        } else {
            r.qb[c] = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.q) + off));
            r.kb[c] = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.k) + off));
            if constexpr (MODE == KDA_GATE_LOG) {
                r.gf[c] = load_f32x4(p.g, off);
            } else {
                r.ab[c] = __ldg(reinterpret_cast<const uint2 *>(static_cast<const uint16_t *>(p.a) + off));
            }
        }
    }
    const uint16_t *vp = static_cast<const uint16_t *>(p.v) + base;
    r.vb[0] = vp[row0];
    r.vb[1] = vp[row0 + 4];
    if constexpr (MODE == KDA_GATE_RAW) {
        r.bb = static_cast<const uint16_t *>(p.b)[t * p.num_heads + h];
    } else {
        r.beta = __ldg(p.beta + t * p.num_heads + h);
    }
}

__device__ __forceinline__ float sum8(float x) {
    x += __shfl_xor_sync(0xffffffffu, x, 1);
    x += __shfl_xor_sync(0xffffffffu, x, 2);
    x += __shfl_xor_sync(0xffffffffu, x, 4);
    return x;
}

template <int D>
__device__ __forceinline__ void unpack4(float *dst, float4 x) {
    dst[0] = x.x; dst[1] = x.y; dst[2] = x.z; dst[3] = x.w;
}

__device__ __forceinline__ void unpack_bf4(float *dst, uint2 x) {
    dst[0] = bf16_lo(x.x); dst[1] = bf16_hi(x.x); dst[2] = bf16_lo(x.y); dst[3] = bf16_hi(x.y);
}

// Store the lane's two rows of the state (k-contiguous layout when FAST).
template <int D, bool FAST>
__device__ __forceinline__ void store_rows(float *base, int64_t sk, int64_t sv, int row0, int sub,
                                           const float (&s)[2][D / 8]) {
    constexpr int NC = D / 32;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const int row = row0 + j * 4;
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int k = c * 32 + sub * 4;
            if constexpr (FAST) {
                *reinterpret_cast<float4 *>(base + static_cast<int64_t>(row) * D + k) =
                    make_float4(s[j][c * 4 + 0], s[j][c * 4 + 1], s[j][c * 4 + 2], s[j][c * 4 + 3]);
            } else {
#pragma unroll
                for (int e = 0; e < 4; ++e) base[row * sv + (k + e) * sk] = s[j][c * 4 + e];
            }
        }
    }
}

// Everything one work item -- (request, head, 32-row value slice) -- needs
// besides its state rows.
struct Item {
    int req, h, v0;
    int64_t bos, eos, slot, tslot, tlen;
    bool rejected;   // valid token range, but a slot failed its bounds check
};

// The op returns its output uninitialised (empty_like) instead of zeroing it
// first (the reference's zeros_like, kda_varlen_recurrent.cpp:142), so with
// `zero_fill` the kernel itself writes zeros where no value is computed: the
// tokens no request covers ([0, cu_seqlens[0]) and [cu_seqlens[num_req], T))
// of the heads processed, and the rows of a request rejected by the bounds
// checks. Threads `gtid` of `gthreads` share the uncovered rows, after their
// items; c0 and cn are cu_seqlens[0] and cu_seqlens[num_req].
template <int D>
__device__ void zero_uncovered(const KdaArgs &p, int64_t c0, int64_t cn, int64_t gtid, int64_t gthreads) {
    if (c0 < 0 || cn > p.num_tokens || c0 > cn) return;   // reported by the items
    const int64_t elems = (c0 + p.num_tokens - cn) * p.head_count * D;
    for (int64_t i = gtid; i < elems; i += gthreads) {
        const int64_t row = i / D, col = i % D;
        const int64_t tr = row / p.head_count;
        const int h = p.head_begin + static_cast<int>(row % p.head_count);
        const int64_t t = tr < c0 ? tr : cn + (tr - c0);
        const int64_t oi = (t * p.num_heads + h) * D + col;
        if (p.out_fp32)
            static_cast<float *>(p.out)[oi] = 0.f;
        else
            static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(0.f);
    }
}
// The output rows of one rejected item (its value slice, every token).
__device__ __forceinline__ void zero_item_rows(const KdaArgs &p, int h, int v0, int64_t bos, int64_t eos, int row0,
                                               int sub, int D) {
    if (sub != 0) return;
    for (int64_t t = bos; t < eos; ++t) {
        const int64_t oi = (t * p.num_heads + h) * D + v0 + row0;
        if (p.out_fp32) {
            static_cast<float *>(p.out)[oi] = 0.f;
            static_cast<float *>(p.out)[oi + 4] = 0.f;
        } else {
            static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(0.f);
            static_cast<__nv_bfloat16 *>(p.out)[oi + 4] = __float2bfloat16_rn(0.f);
        }
    }
}

// Decodes item `it` and checks its metadata; false (with the status word set)
// when the request must be skipped. Identical in every thread of the CTA.
__device__ __forceinline__ bool decode_item(const KdaArgs &p, int64_t it, int nslice, Item &m) {
    m.v0 = static_cast<int>(it % nslice) * kBV;
    it /= nslice;
    m.h = p.head_begin + static_cast<int>(it % p.head_count);
    m.req = static_cast<int>(it / p.head_count);
    m.bos = load_index(p.cu_seqlens, p.index_bytes[1], m.req);
    m.eos = load_index(p.cu_seqlens, p.index_bytes[1], m.req + 1);
    m.slot = load_index(p.indices, p.index_bytes[0], m.req);
    m.tslot = 0;
    m.tlen = -1;
    m.rejected = false;
    if (m.bos < 0 || m.eos < m.bos || m.eos > p.num_tokens) {
        if (threadIdx.x == 0) report(p.status, KDA_DEVICE_ERR_BAD_SEQLENS);
        return false;
    }
    if (m.slot < 0 || m.slot >= p.num_slots) {
        if (threadIdx.x == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
        m.rejected = true;
        return false;
    }
    if (p.track_indices != nullptr) {
        m.tslot = load_index(p.track_indices, p.index_bytes[2], m.req);
        if (m.tslot < 0 || m.tslot >= p.num_slots) {
            if (threadIdx.x == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
            m.rejected = true;
            return false;
        }
        if (m.tslot > 0) m.tlen = load_index(p.track_lens, p.index_bytes[3], m.req);
    }
    return true;
}

// The token loop of one item with the state rows already in registers:
// prologue, recurrence step, output, prefix/per-step checkpoints, final
// write-back (kda_python.py:271-307).
// `cur` holds the item's first token when `staged` (read from a ring stage by
// the caller); otherwise it is loaded here.
// The raw gate's per-head parameters a lane needs: A_log[h] and the four
// dt_bias entries of its own key group (group (lane / 8) % (D / 32), keys
// group * 32 + sub * 4 .. + 3), loaded ahead of use by the caller.
struct RawGateParams {
    float4 dtb;
    float a_log;
};
// The loads are volatile asm so the compiler issues them where they are
// written (one item ahead) instead of sinking them next to their first use.
template <int D>
__device__ __forceinline__ RawGateParams load_raw_params(const KdaArgs &p, int h, int sub) {
    const int grp = ((threadIdx.x & 31) >> 3) % (D / 32);
    RawGateParams r;
    const float *d = p.dt_bias + h * D + grp * 32 + sub * 4;
    asm volatile("ld.global.nc.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(r.dtb.x), "=f"(r.dtb.y), "=f"(r.dtb.z), "=f"(r.dtb.w)
                 : "l"(d));
    asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(r.a_log) : "l"(p.A_log + h));
    return r;
}

template <int D, int MODE, bool FAST>
__device__ __forceinline__ void run_item(const KdaArgs &p, const Item &m, float (&s)[2][D / 8], int row0, int sub,
                                         TokenRaw<D, MODE> &cur, bool staged, const RawGateParams &rp) {
    constexpr int NC = D / 32;
    constexpr int NE = D / 8;
    const int h = m.h, v0 = m.v0;
    const int64_t sk = p.state_stride[2], sv = p.state_stride[3];
    const int64_t row_off = FAST ? static_cast<int64_t>(v0) * D : v0 * sv;

    // Raw gate: the decay of a key depends on (token, head, key) only, so the
    // four 8-lane row groups of a warp split the key groups between them
    // (group (lane / 8) % NC), compute their decays once and share them by
    // shuffles, instead of each lane evaluating all of its D / 8 keys.
    const int grp = ((threadIdx.x & 31) >> 3) % NC;
    float expA = 0.f;
    if constexpr (MODE == KDA_GATE_RAW) expA = expf(rp.a_log);

    float *const track_state =
        (m.tslot > 0) ? p.state + m.tslot * p.state_stride[0] + h * p.state_stride[1] + row_off : nullptr;
    if (m.tslot > 0 && m.tlen == 0) store_rows<D, FAST>(track_state, sk, sv, row0, sub, s);

    float *const mid_head =
        (p.intermediate != nullptr && m.slot > 0)
            ? p.intermediate + m.req * p.mid_stride[0] + h * p.mid_stride[2] +
                  (FAST ? static_cast<int64_t>(v0) * D : v0 * p.mid_stride[4])
            : nullptr;

    TokenRaw<D, MODE> nxt;
    if (m.bos < m.eos && !staged) load_token<D, MODE>(cur, p, m.bos, h, sub, v0 + row0);

    for (int64_t t = m.bos; t < m.eos; ++t) {
        if (t + 1 < m.eos) load_token<D, MODE>(nxt, p, t + 1, h, sub, v0 + row0);

        // ---- prologue: norms, decay, beta (kda_python.py:26-38) ----
        float qn[NE], kn[NE], dec[NE];
        float beta;
        if constexpr (MODE == KDA_GATE_PREPARED) {
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                unpack4<D>(qn + c * 4, cur.qf[c]);
                unpack4<D>(kn + c * 4, cur.kf[c]);
                unpack4<D>(dec + c * 4, cur.gf[c]);
            }
            beta = cur.beta;
        } else {
            float q[NE], k[NE];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                unpack_bf4(q + c * 4, cur.qb[c]);
                unpack_bf4(k + c * 4, cur.kb[c]);
            }
            // Two partial sums per reduction (even / odd elements): shorter
            // dependent chains for the latency-bound item loop.
            float sq0 = 0.f, sq1 = 0.f, sk0 = 0.f, sk1 = 0.f;
#pragma unroll
            for (int e = 0; e < NE; e += 2) {
                sq0 = fmaf(q[e], q[e], sq0);
                sq1 = fmaf(q[e + 1], q[e + 1], sq1);
                sk0 = fmaf(k[e], k[e], sk0);
                sk1 = fmaf(k[e + 1], k[e + 1], sk1);
            }
            const float sq = sum8(sq0 + sq1);
            const float sk2 = sum8(sk0 + sk1);
            // One reciprocal per row instead of a division per element; the
            // product differs from q / ||q|| by at most an ulp.
            const float rq = p.scale / sqrtf(sq + kNormEps), rk = 1.0f / sqrtf(sk2 + kNormEps);
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                qn[e] = q[e] * rq;
                kn[e] = k[e] * rk;
            }
            if constexpr (MODE == KDA_GATE_LOG) {
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    float g4[4];
                    unpack4<D>(g4, cur.gf[c]);
#pragma unroll
                    for (int e = 0; e < 4; ++e) dec[c * 4 + e] = expf(g4[e]);
                }
                beta = cur.beta;
            } else {
                uint2 ab = cur.ab[0];
#pragma unroll
                for (int c = 1; c < NC; ++c)
                    if (grp == c) ab = cur.ab[c];
                float a4[4], mine[4];
                unpack_bf4(a4, ab);
                const float dtb[4] = {rp.dtb.x, rp.dtb.y, rp.dtb.z, rp.dtb.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float gate = expA * (a4[e] + dtb[e]);
                    mine[e] = expf(p.lower_bound * sigmoidf_(gate));
                }
#pragma unroll
                for (int c = 0; c < NC; ++c)
#pragma unroll
                    for (int e = 0; e < 4; ++e) dec[c * 4 + e] = __shfl_sync(0xffffffffu, mine[e], c * 8 + sub);
                beta = sigmoidf_(__uint_as_float(static_cast<uint32_t>(cur.bb) << 16));
            }
        }

        // ---- recurrence step ----
        float pa[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int e = 0; e < NE; e += 2) {
                s[j][e] *= dec[e];
                s[j][e + 1] *= dec[e + 1];
                a0 = fmaf(s[j][e], kn[e], a0);
                a1 = fmaf(s[j][e + 1], kn[e + 1], a1);
            }
            pa[j] = a0 + a1;
        }
        pa[0] = sum8(pa[0]);
        pa[1] = sum8(pa[1]);
        float po[2];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float vv = __uint_as_float(static_cast<uint32_t>(cur.vb[j]) << 16);
            const float d = (vv - pa[j]) * beta;
            float a0 = 0.f, a1 = 0.f;
#pragma unroll
            for (int e = 0; e < NE; e += 2) {
                s[j][e] = fmaf(kn[e], d, s[j][e]);
                s[j][e + 1] = fmaf(kn[e + 1], d, s[j][e + 1]);
                a0 = fmaf(s[j][e], qn[e], a0);
                a1 = fmaf(s[j][e + 1], qn[e + 1], a1);
            }
            po[j] = a0 + a1;
        }
        po[0] = sum8(po[0]);
        po[1] = sum8(po[1]);
        if (sub == 0) {
            const int64_t oi = (t * p.num_heads + h) * D + v0 + row0;
            if (p.out_fp32) {
                float *o = static_cast<float *>(p.out) + oi;
                o[0] = po[0];
                o[4] = po[1];
            } else {
                __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + oi;
                o[0] = __float2bfloat16_rn(po[0]);
                o[4] = __float2bfloat16_rn(po[1]);
            }
        }
        const int64_t step = t - m.bos;
        if (m.tslot > 0 && step + 1 == m.tlen) store_rows<D, FAST>(track_state, sk, sv, row0, sub, s);
        if (mid_head != nullptr)
            store_rows<D, FAST>(mid_head + step * p.mid_stride[1], p.mid_stride[3], p.mid_stride[4], row0, sub, s);
        cur = nxt;
    }

    if (p.intermediate == nullptr && m.slot > 0) {
        float *head_state = p.state + m.slot * p.state_stride[0] + h * p.state_stride[1] + row_off;
        store_rows<D, FAST>(head_state, sk, sv, row0, sub, s);
    }
}

// Production layout (K-contiguous, 16-byte aligned): persistent CTAs walk the
// items with a STAGES-deep ring. Thread 0 fills a ring stage with everything
// an item needs -- its 32 x D state rows and, when the token pointers are
// 16-byte aligned, its first token's q, k, gate rows and v slice, all by bulk
// TMA copies on the stage's mbarrier -- plus a header with the item's
// metadata; it reads the next item's cu_seqlens and slot one refill ahead, and
// the compute threads read beta one item ahead, so no global-memory round
// trip sits between an item's stage landing and its arithmetic. Item n of a
// CTA uses stage n % STAGES, whose mbarrier completes phase (n / STAGES) & 1.
struct StageMeta {
    int64_t bos, eos, slot, tslot, tlen;
    int req, h, v0, ok;
    uint32_t bword;   // beta (or the 4-byte word holding the raw b) of the first token
    int bsel;         // 0: not staged (load it); 1: bword / its low half; 2: its high half
    float a_log;      // raw gate: A_log[h]
};
template <int D, int MODE>
struct RingStage {
    static constexpr int QE = MODE == KDA_GATE_PREPARED ? 4 : 2;   // q, k element bytes
    static constexpr int GE = MODE == KDA_GATE_RAW ? 2 : 4;        // gate row element bytes (a or g)
    static constexpr int kQ = kBV * D * 4;                         // after the state rows
    static constexpr int kK = kQ + D * QE;
    static constexpr int kG = kK + D * QE;
    static constexpr int kV = kG + D * GE;                         // bf16 v slice (kBV values)
    static constexpr int kTokBytes = kV + kBV * 2 - kQ;
    // raw gate: the item's head's dt_bias row (D fp32), copied with the tiles
    static constexpr int kDtb = (kV + kBV * 2 + 15) / 16 * 16;
    static constexpr int kDtbBytes = MODE == KDA_GATE_RAW ? D * 4 : 0;
    static constexpr int kMeta = kDtb + kDtbBytes;
    static constexpr int kBytes = (kMeta + static_cast<int>(sizeof(StageMeta)) + 127) / 128 * 128;
};

// The first token of an item from its ring stage (beta from the header, or a
// global load when the producer could not stage it).
template <int D, int MODE>
__device__ __forceinline__ void token_from_stage(TokenRaw<D, MODE> &r, const KdaArgs &p, const unsigned char *stage,
                                                 const StageMeta &sm, int sub, int row0) {
    using RS = RingStage<D, MODE>;
    constexpr int NC = D / 32;
#pragma unroll
    for (int c = 0; c < NC; ++c) {
        const int e = c * 32 + sub * 4;
        if constexpr (MODE == KDA_GATE_PREPARED) {
            r.qf[c] = *reinterpret_cast<const float4 *>(stage + RS::kQ + e * 4);
            r.kf[c] = *reinterpret_cast<const float4 *>(stage + RS::kK + e * 4);
            r.gf[c] = *reinterpret_cast<const float4 *>(stage + RS::kG + e * 4);
        } else {
            r.qb[c] = *reinterpret_cast<const uint2 *>(stage + RS::kQ + e * 2);
            r.kb[c] = *reinterpret_cast<const uint2 *>(stage + RS::kK + e * 2);
            if constexpr (MODE == KDA_GATE_LOG)
                r.gf[c] = *reinterpret_cast<const float4 *>(stage + RS::kG + e * 4);
            else
                r.ab[c] = *reinterpret_cast<const uint2 *>(stage + RS::kG + e * 2);
        }
    }
    const uint16_t *vs = reinterpret_cast<const uint16_t *>(stage + RS::kV);
    r.vb[0] = vs[row0];
    r.vb[1] = vs[row0 + 4];
    const int64_t bi = sm.bos * p.num_heads + sm.h;
    if constexpr (MODE == KDA_GATE_RAW)
        r.bb = sm.bsel == 0 ? static_cast<const uint16_t *>(p.b)[bi]
                            : static_cast<uint16_t>(sm.bsel == 1 ? sm.bword & 0xffffu : sm.bword >> 16);
    else
        r.beta = sm.bsel == 0 ? __ldg(p.beta + bi) : __uint_as_float(sm.bword);
}

// One producer warp per CTA refills the ring; the compute warps never wait for
// a refill or for one another. Stage n % STAGES: `full` completes when its
// copies (and the beta word) have landed, `empty` when all four compute warps
// have read it.
template <int D, int MODE, int STAGES, int MINB>
__global__ void __launch_bounds__(kRecThreads + 32, MINB)
recurrent_ring_kernel(const KdaArgs p, int nslice, int64_t num_items, int tok_bulk, int32_t len_lo,
                      int32_t len_hi, int zero_fill) {
    using RS = RingStage<D, MODE>;
    constexpr int NC = D / 32;
    constexpr uint32_t kTileBytes = kBV * D * sizeof(float);
    extern __shared__ __align__(128) unsigned char ring[];    // STAGES x RS::kBytes
    __shared__ __align__(8) uint64_t full[STAGES];
    __shared__ __align__(8) uint64_t empty[STAGES];

    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int sub = lane & 7, rq = lane >> 3;
    const int row0 = warp * kRowsPerWarp + rq;
    const int64_t first = blockIdx.x, stride = gridDim.x;
    auto meta_of = [&](int st) { return reinterpret_cast<StageMeta *>(ring + st * RS::kBytes + RS::kMeta); };

    if (tid == 0) {
#pragma unroll
        for (int st = 0; st < STAGES; ++st) {
            mbar_init(&full[st], 1);
            mbar_init(&empty[st], kRecThreads / 32);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kRecThreads / 32) {
        // ===== producer =====
        if (lane != 0) return;
        int st = 0;
        uint32_t use = 0;   // how many times stage st has been filled
        for (int64_t it = first; it < num_items; it += stride) {
            if (use > 0 && !mbar_wait(&empty[st], (use - 1) & 1u, p.status)) return;
            unsigned char *stage = ring + st * RS::kBytes;
            StageMeta *hdr = meta_of(st);
            const int64_t x = it / nslice;
            const int h = p.head_begin + static_cast<int>(x % p.head_count);
            const int req = static_cast<int>(x / p.head_count);
            const int v0 = static_cast<int>(it % nslice) * kBV;
            const int64_t bos = load_index(p.cu_seqlens, p.index_bytes[1], req);
            const int64_t eos = load_index(p.cu_seqlens, p.index_bytes[1], req + 1);
            const int64_t slot = load_index(p.indices, p.index_bytes[0], req);
            int ok = 1, zero = 0;
            int64_t tslot = 0, tlen = -1;
            if (bos < 0 || eos < bos || eos > p.num_tokens) {
                report(p.status, KDA_DEVICE_ERR_BAD_SEQLENS);
                ok = 0;
            } else if (slot < 0 || slot >= p.num_slots) {
                report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
                ok = 0;
                zero = zero_fill;
            } else if (p.track_indices != nullptr) {
                tslot = load_index(p.track_indices, p.index_bytes[2], req);
                if (tslot < 0 || tslot >= p.num_slots) {
                    report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
                    ok = 0;
                    zero = zero_fill;
                } else if (tslot > 0) {
                    tlen = load_index(p.track_lens, p.index_bytes[3], req);
                }
            }
            // A request outside [len_lo, len_hi] belongs to another kernel of
            // the same launch: nothing is read or written for it here.
            if (eos - bos < len_lo || eos - bos > len_hi) ok = zero = 0;
            // beta (raw b) of the first token into the header by a 4-byte
            // cp.async that the stage's barrier also waits for (its tracking
            // arrive precedes the expect-tx arrive, so the phase cannot
            // complete without it). The raw b is 2 bytes: its aligned word is
            // copied only when that word lies inside the tensor.
            const char *bsrc = nullptr;
            int bsel = 0;
            if (ok && bos < eos) {
                const int64_t bi = bos * p.num_heads + h;
                if constexpr (MODE == KDA_GATE_RAW) {
                    if ((bi | 1) < static_cast<int64_t>(p.num_tokens) * p.num_heads) {
                        bsrc = reinterpret_cast<const char *>(static_cast<const uint16_t *>(p.b) + (bi & ~int64_t(1)));
                        bsel = 1 + static_cast<int>(bi & 1);
                    }
                } else {
                    bsrc = reinterpret_cast<const char *>(p.beta + bi);
                    bsel = 1;
                }
            }
            hdr->bos = bos;
            hdr->eos = eos;
            hdr->slot = slot;
            hdr->tslot = tslot;
            hdr->tlen = tlen;
            hdr->req = req;
            hdr->h = h;
            hdr->v0 = v0;
            hdr->ok = ok;
            hdr->bsel = bsel;   // bword is written only by the copy below
            // A rejected request's output rows: zeros, written here by the
            // producer thread (a rare path the compute warps never see).
            if (zero) {
                for (int64_t t = bos; t < eos; ++t)
                    for (int r = 0; r < kBV; ++r) {
                        const int64_t oi = (t * p.num_heads + h) * D + v0 + r;
                        if (p.out_fp32)
                            static_cast<float *>(p.out)[oi] = 0.f;
                        else
                            static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(0.f);
                    }
            }
            if constexpr (MODE == KDA_GATE_RAW) hdr->a_log = ok ? __ldg(p.A_log + h) : 0.f;
            if (bsrc != nullptr) {
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(&hdr->bword)), "l"(bsrc)
                             : "memory");
                asm volatile("cp.async.mbarrier.arrive.shared::cta.b64 [%0];" ::"r"(smem_addr(&full[st]))
                             : "memory");
            }
            const bool st_in = ok && slot > 0;
            const bool tk_in = ok && tok_bulk && bos < eos;
            const bool dt_in = MODE == KDA_GATE_RAW && ok;
            const uint32_t bytes = (st_in ? kTileBytes : 0u) + (tk_in ? static_cast<uint32_t>(RS::kTokBytes) : 0u) +
                                   (dt_in ? static_cast<uint32_t>(RS::kDtbBytes) : 0u);
            if (bytes > 0) {
                mbar_arrive_expect_tx(&full[st], bytes);
                if (dt_in) bulk_g2s(stage + RS::kDtb, p.dt_bias + static_cast<int64_t>(h) * D, RS::kDtbBytes, &full[st]);
                if (st_in)
                    bulk_g2s(stage, p.state + slot * p.state_stride[0] + h * p.state_stride[1] + static_cast<int64_t>(v0) * D,
                             kTileBytes, &full[st]);
                if (tk_in) {
                    const int64_t row = bos * p.num_heads + h;
                    const uint8_t *gsrc = MODE == KDA_GATE_RAW ? static_cast<const uint8_t *>(p.a)
                                                               : reinterpret_cast<const uint8_t *>(p.g);
                    bulk_g2s(stage + RS::kQ, static_cast<const uint8_t *>(p.q) + row * D * RS::QE, D * RS::QE,
                             &full[st]);
                    bulk_g2s(stage + RS::kK, static_cast<const uint8_t *>(p.k) + row * D * RS::QE, D * RS::QE,
                             &full[st]);
                    bulk_g2s(stage + RS::kG, gsrc + row * D * RS::GE, D * RS::GE, &full[st]);
                    bulk_g2s(stage + RS::kV, static_cast<const uint8_t *>(p.v) + (row * D + v0) * 2, kBV * 2,
                             &full[st]);
                }
            } else {
                mbar_arrive(&full[st]);
            }
            if (++st == STAGES) {
                st = 0;
                ++use;
            }
        }
        // Tokens no request covers (normally none): the last CTA's producer.
        if (zero_fill && blockIdx.x == gridDim.x - 1)
            zero_uncovered<D>(p, load_index(p.cu_seqlens, p.index_bytes[1], 0),
                              load_index(p.cu_seqlens, p.index_bytes[1], p.num_req), 0, 1);
        return;
    }

    // ===== compute warps =====
    int st = 0;
    uint32_t phase = 0;
    for (int64_t it = first; it < num_items; it += stride) {
        if (!mbar_wait(&full[st], phase, p.status)) return;
        const unsigned char *stage = ring + st * RS::kBytes;
        const StageMeta sm = *meta_of(st);
        Item m;
        m.req = sm.req;
        m.h = sm.h;
        m.v0 = sm.v0;
        m.bos = sm.bos;
        m.eos = sm.eos;
        m.slot = sm.slot;
        m.tslot = sm.tslot;
        m.tlen = sm.tlen;
        const bool ok = sm.ok != 0;
        float s[2][D / 8];
        if (ok && m.slot > 0) {
            const float *tile = reinterpret_cast<const float *>(stage);
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    unpack4<D>(&s[j][c * 4],
                               *reinterpret_cast<const float4 *>(&tile[(row0 + j * 4) * D + c * 32 + sub * 4]));
        } else {
#pragma unroll
            for (int j = 0; j < 2; ++j)
#pragma unroll
                for (int e = 0; e < D / 8; ++e) s[j][e] = 0.f;
        }
        TokenRaw<D, MODE> cur;
        const bool staged = ok && tok_bulk && m.bos < m.eos;
        if (staged) token_from_stage<D, MODE>(cur, p, stage, sm, sub, row0);
        // Raw gate: the head's A_log (header) and this lane's dt_bias group
        // (copied into the stage with the tiles).
        RawGateParams rp{};
        if constexpr (MODE == KDA_GATE_RAW) {
            if (ok) {
                const int grp = rq % (D / 32);
                rp.dtb = *reinterpret_cast<const float4 *>(stage + RS::kDtb + (grp * 32 + sub * 4) * 4);
                rp.a_log = sm.a_log;
            }
        }
        // This warp is done with the stage.
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        if (ok) run_item<D, MODE, true>(p, m, s, row0, sub, cur, staged, rp);
        if (++st == STAGES) {
            st = 0;
            phase ^= 1u;
        }
    }
}

// Any other pool layout: one CTA per item, strided loads straight from the
// pool (used by prepared_recurrent on a [K,V]-contiguous state).
template <int D, int MODE>
__global__ void __launch_bounds__(kRecThreads, 3)
recurrent_strided_kernel(const KdaArgs p, int nslice, int32_t len_lo, int32_t len_hi, int zero_fill) {
    constexpr int NE = D / 8;
    const int tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int sub = lane & 7, rq = lane >> 3;
    const int row0 = warp * kRowsPerWarp + rq;
    int64_t c0 = 0, cn = 0;
    if (zero_fill) {
        c0 = load_index(p.cu_seqlens, p.index_bytes[1], 0);
        cn = load_index(p.cu_seqlens, p.index_bytes[1], p.num_req);
    }
    auto finish = [&] {
        if (zero_fill)
            zero_uncovered<D>(p, c0, cn, static_cast<int64_t>(blockIdx.x) * kRecThreads + tid,
                              static_cast<int64_t>(gridDim.x) * kRecThreads);
    };
    Item m;
    const bool valid = decode_item(p, blockIdx.x, nslice, m);
    if (m.eos - m.bos < len_lo || m.eos - m.bos > len_hi) return finish();   // another kernel's request
    if (!valid) {
        if (zero_fill && m.rejected) zero_item_rows(p, m.h, m.v0, m.bos, m.eos, row0, sub, D);
        return finish();
    }
    const int64_t sk = p.state_stride[2], sv = p.state_stride[3];
    float s[2][NE];
    if (m.slot > 0) {
        const float *hs = p.state + m.slot * p.state_stride[0] + m.h * p.state_stride[1];
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < NE; ++e) {
                const int k = (e >> 2) * 32 + sub * 4 + (e & 3);
                s[j][e] = hs[(m.v0 + row0 + j * 4) * sv + k * sk];
            }
    } else {
#pragma unroll
        for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < NE; ++e) s[j][e] = 0.f;
    }
    TokenRaw<D, MODE> cur;
    RawGateParams rp{};
    if constexpr (MODE == KDA_GATE_RAW) rp = load_raw_params<D>(p, m.h, sub);
    run_item<D, MODE, false>(p, m, s, row0, sub, cur, false, rp);
    finish();
}

// ---------------------------------------------------------------------------
// Host side: validation and dispatch
// ---------------------------------------------------------------------------

static bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static int validate_common(const KdaArgs *a) {
    if (a == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (a->head_dim != 64 && a->head_dim != 128) return KDA_ERR_UNSUPPORTED;
    if (a->num_req < 0 || a->num_tokens < 0 || a->num_heads <= 0) return KDA_ERR_INVALID_ARGUMENT;
    if (a->head_begin < 0 || a->head_count < 0 || a->head_begin + a->head_count > a->num_heads)
        return KDA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 4; ++i)
        if (a->index_bytes[i] != 4 && a->index_bytes[i] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (a->num_req == 0 || a->head_count == 0) return KDA_OK;
    if (a->state == nullptr || a->num_slots <= 0 || a->indices == nullptr || a->cu_seqlens == nullptr ||
        a->out == nullptr || a->v == nullptr || a->q == nullptr || a->k == nullptr)
        return KDA_ERR_INVALID_ARGUMENT;
    if ((a->track_indices == nullptr) != (a->track_lens == nullptr)) return KDA_ERR_INVALID_ARGUMENT;
    switch (a->gate_mode) {
        case KDA_GATE_RAW:
            if (a->a == nullptr || a->b == nullptr || a->A_log == nullptr || a->dt_bias == nullptr)
                return KDA_ERR_INVALID_ARGUMENT;
            break;
        case KDA_GATE_LOG:
        case KDA_GATE_PREPARED:
            if (a->g == nullptr || a->beta == nullptr) return KDA_ERR_INVALID_ARGUMENT;
            break;
        default:
            return KDA_ERR_INVALID_ARGUMENT;
    }
    // Four-element vector loads: bf16 rows need 8-byte, fp32 rows 16-byte
    // alignment of the base pointer (row offsets are multiples of 4 elements).
    auto aligned8 = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 7u) == 0; };
    if (a->gate_mode == KDA_GATE_PREPARED) {
        if (!aligned16(a->q) || !aligned16(a->k) || !aligned16(a->g)) return KDA_ERR_ALIGNMENT;
    } else {
        if (!aligned8(a->q) || !aligned8(a->k)) return KDA_ERR_ALIGNMENT;
        if (a->gate_mode == KDA_GATE_LOG && !aligned16(a->g)) return KDA_ERR_ALIGNMENT;
        if (a->gate_mode == KDA_GATE_RAW && (!aligned8(a->a) || !aligned16(a->dt_bias)))
            return KDA_ERR_ALIGNMENT;
    }
    return KDA_OK;
}

// The state slice is one contiguous, 16-byte aligned run of kBV rows.
static bool state_fast(const KdaArgs *a) {
    const int64_t D = a->head_dim;
    return aligned16(a->state) && a->state_stride[2] == 1 && a->state_stride[3] == D &&
           a->state_stride[0] % 4 == 0 && a->state_stride[1] % 4 == 0;
}

static bool mid_fast(const KdaArgs *a) {
    if (a->intermediate == nullptr) return true;
    const int64_t D = a->head_dim;
    return aligned16(a->intermediate) && a->mid_stride[3] == 1 && a->mid_stride[4] == D &&
           a->mid_stride[0] % 4 == 0 && a->mid_stride[1] % 4 == 0 && a->mid_stride[2] % 4 == 0;
}

// Ring depth and resident CTAs per SM: four compute warps and a producer
// warp per CTA at up to 168 registers allow two CTAs per SM (three would cap
// registers at 136 and spill); shared memory then holds six 17 KiB stages per
// CTA.
template <int MODE>
struct RingShape {
    static constexpr int kStages = 6;
    static constexpr int kMinBlocks = 2;
};

struct DeviceInfo {
    int sms = 0;
};

static int sm_count() {
    static DeviceInfo info[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (info[dev].sms == 0) {
        int sms = 0;
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        info[dev].sms = sms > 0 ? sms : 148;
    }
    return info[dev].sms;
}

template <int D, int MODE>
static void launch_rec(const KdaArgs *a, bool fast, cudaStream_t st, int32_t len_lo, int32_t len_hi, int zero_fill) {
    const int nslice = D / kBV;
    const int64_t items = static_cast<int64_t>(a->num_req) * a->head_count * nslice;
    if (fast) {
        constexpr size_t smem = static_cast<size_t>(RingShape<MODE>::kStages) * RingStage<D, MODE>::kBytes;
        // Per device: opt in to the dynamic shared memory once and cache the
        // resident-CTA count the grid is sized from (a multiple of the SMs).
        static int per_sm[64];
        int dev = 0;
        cudaGetDevice(&dev);
        dev = (dev >= 0 && dev < 64) ? dev : 0;
        if (per_sm[dev] == 0) {
            cudaFuncSetAttribute(recurrent_ring_kernel<D, MODE, RingShape<MODE>::kStages, RingShape<MODE>::kMinBlocks>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
            int n = 0;
            cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, recurrent_ring_kernel<D, MODE, RingShape<MODE>::kStages, RingShape<MODE>::kMinBlocks>,
                                                          kRecThreads + 32, smem);
            per_sm[dev] = n > 0 ? n : 1;
        }
        const int64_t cap = static_cast<int64_t>(sm_count()) * per_sm[dev];
        const int64_t grid = items < cap ? items : cap;
        // The token rows ride along with the state tile when every token
        // pointer allows a bulk copy (16-byte aligned rows).
        const void *gate = MODE == KDA_GATE_RAW ? static_cast<const void *>(a->a) : static_cast<const void *>(a->g);
        const int tok_bulk = aligned16(a->q) && aligned16(a->k) && aligned16(gate) && aligned16(a->v) ? 1 : 0;
        recurrent_ring_kernel<D, MODE, RingShape<MODE>::kStages, RingShape<MODE>::kMinBlocks>
            <<<static_cast<unsigned>(grid), kRecThreads + 32, smem, st>>>(*a, nslice, items, tok_bulk, len_lo, len_hi, zero_fill);
    } else {
        recurrent_strided_kernel<D, MODE>
            <<<static_cast<unsigned>(items), kRecThreads, 0, st>>>(*a, nslice, len_lo, len_hi, zero_fill);
    }
}

template <int D>
static void dispatch_mode(const KdaArgs *a, bool fast, cudaStream_t st, int32_t len_lo, int32_t len_hi,
                          int zero_fill) {
    switch (a->gate_mode) {
        case KDA_GATE_RAW: launch_rec<D, KDA_GATE_RAW>(a, fast, st, len_lo, len_hi, zero_fill); break;
        case KDA_GATE_LOG: launch_rec<D, KDA_GATE_LOG>(a, fast, st, len_lo, len_hi, zero_fill); break;
        default: launch_rec<D, KDA_GATE_PREPARED>(a, fast, st, len_lo, len_hi, zero_fill); break;
    }
}

// The recurrence over the requests of length len_lo..len_hi only (the others
// are left untouched): the chunk prefill hands its shortest requests to this
// kernel, where a token costs a step rather than a 64-row chunk.
int recurrent_launch_range(const KdaArgs *args, int32_t len_lo, int32_t len_hi, cudaStream_t st) {
    const int rc = validate_common(args);
    if (rc != KDA_OK) return rc;
    if (args->num_req == 0 || args->head_count == 0) return KDA_OK;
    const bool fast = state_fast(args) && mid_fast(args);
    if (args->head_dim == 128)
        dispatch_mode<128>(args, fast, st, len_lo, len_hi, 0);
    else
        dispatch_mode<64>(args, fast, st, len_lo, len_hi, 0);
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}

}  // namespace kda

extern "C" int kda_abi_version(void) { return KDA_ABI_VERSION; }

extern "C" const char *kda_status_string(int code) {
    switch (code) {
        case KDA_OK: return "ok";
        case KDA_ERR_INVALID_ARGUMENT: return "invalid argument";
        case KDA_ERR_UNSUPPORTED: return "unsupported configuration";
        case KDA_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
        case KDA_ERR_WORKSPACE: return "workspace missing or too small";
        case KDA_ERR_LAUNCH: return "CUDA launch failed";
        case KDA_ERR_TOO_LARGE: return "batch beyond the fixed in-library scratch capacity";
        case KDA_DEVICE_ERR_WAIT_TIMEOUT: return "device: bounded mbarrier wait expired";
        case KDA_DEVICE_ERR_BAD_SLOT: return "device: state slot index out of range";
        case KDA_DEVICE_ERR_BAD_SEQLENS: return "device: cu_seqlens not monotone or beyond T";
        case KDA_DEVICE_ERR_GATE_RANGE: return "device: gate span beyond the chunk kernel's exponent range";
        default: return "unknown status";
    }
}

namespace kda {
// Every request; with `zero_fill` the output rows no value is computed for
// are written as zeros (kda_recurrent_launch); prepared_recurrent's output is
// the caller's tensor and keeps its other rows.
static int recurrent_launch_all(const KdaArgs *args, cudaStream_t st, int zero_fill) {
    const int rc = validate_common(args);
    if (rc != KDA_OK) return rc;
    if (args->num_req == 0 || args->head_count == 0) return KDA_OK;
    const bool fast = state_fast(args) && mid_fast(args);
    if (args->head_dim == 128)
        dispatch_mode<128>(args, fast, st, 0, INT32_MAX, zero_fill);
    else
        dispatch_mode<64>(args, fast, st, 0, INT32_MAX, zero_fill);
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
}  // namespace kda

extern "C" int kda_recurrent_launch(const KdaArgs *args, void *stream) {
    return kda::recurrent_launch_all(args, static_cast<cudaStream_t>(stream), 1);
}

extern "C" int kda_prepared_recurrent_launch(const KdaArgs *args, void *stream) {
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    KdaArgs a = *args;
    a.gate_mode = KDA_GATE_PREPARED;
    a.intermediate = nullptr;
    return kda::recurrent_launch_all(&a, static_cast<cudaStream_t>(stream), 0);
}
