// Chunk-64 WY/UT prefill of the GLM KDA operator on sm_100a, behind
// kda_chunk_launch / kda_chunk_workspace_bytes.
//
// Math per chunk of BT = 64 tokens (kda_python.py:121-182; reference kernel
// sgl-glm53-ascend-ops/csrc/kda/chunk/kda_varlen_chunk_kernel.cpp):
//   gc   = cumsum(g) within the chunk                      [64 x D]
//   A'   = beta_i sum_k kn_i kn_j e^{gc_i - gc_j}   (j < i) [64 x 64]
//   Aqk  = sum_k qn_i kn_j e^{gc_i - gc_j}          (j <= i)
//   T    = (I + A')^-1,  TB = T diag(beta)
//   W    = TB (kn e^{gc}),   u = TB v
//   v'   = u - W S,   o = (qn e^{gc}) S + Aqk v'
//   S   <- e^{gc_last} S + (kn e^{gc_last - gc})^T v'
//
// B200 design (no counterpart in the reference):
//   * one CTA per (sequence, head), 8 warps, the whole chunk loop in one CTA;
//     requests are visited longest-first (a one-block prologue kernel writes
//     the order into the workspace).
//   * tensor-core products use mma.sync bf16 with every inexact fp32 operand
//     split into hi + lo bf16 and three products (hi.hi + hi.lo + lo.hi):
//     plain bf16 operands miss the output bar (5e-3 of the output RMS) by
//     3-13x on these inputs, the split form lands at ~2e-4.
//   * the exponent range is handled with 16-row blocks anchored at their
//     midpoint row m_I: X = kn e^{gc - m_I}, Y = qn e^{gc - m_I} and
//     Z = kn e^{m_I - gc} stay within e^{+-8|g|}, and a block pair (I, J)
//     is X_I (e^{m_I - m_J}) Z_J^T with the factor <= 1 (fp32 exp overflows at
//     e^88.7; the reference rebases per 32 rows for the same reason,
//     kda_varlen_chunk.h:24-29).
//   * the state lives transposed (S^T, value rows x key columns, the pool's
//     own [V][K] order) in registers: warp w owns value rows [16w, 16w+16) as
//     mma C fragments, which feed the next product directly as A fragments;
//     B operands come from swizzled bf16 hi/lo tiles through ldmatrix.
//   * the next chunk's q/k/g (and v) are fetched with cp.async while the W
//     product and the state scan of this chunk run.
//   * any sequence length: a partial last chunk is zero-filled (k = q = v =
//     g = beta = 0), which leaves the state and the real rows unchanged.

#include "kda_common.cuh"

#include <mutex>

namespace kda {
namespace chunk {

constexpr int BT = 64;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// ---------------------------------------------------------------------------
// mma.sync / ldmatrix / cp.async primitives
// ---------------------------------------------------------------------------

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t b0,
                                         const uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// hi.hi + hi.lo + lo.hi: the split-bf16 product (lo.lo is below fp32 noise).
__device__ __forceinline__ void mma3(float (&d)[4], const uint32_t (&ah)[4], const uint32_t (&al)[4],
                                     uint32_t bh0, uint32_t bh1, uint32_t bl0, uint32_t bl1) {
    mma16816(d, al, bh0, bh1);
    mma16816(d, ah, bl0, bl1);
    mma16816(d, ah, bh0, bh1);
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_addr(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Pack two floats as bf16x2 (x0 in the low half) and the residual pair.
__device__ __forceinline__ uint32_t pack_bf16(float x0, float x1) {
    __nv_bfloat162 v = __floats2bfloat162_rn(x0, x1);
    return *reinterpret_cast<uint32_t *>(&v);
}
__device__ __forceinline__ void split2(float x0, float x1, uint32_t &hi, uint32_t &lo) {
    hi = pack_bf16(x0, x1);
    lo = pack_bf16(x0 - bf16_lo(hi), x1 - bf16_hi(hi));
}
__device__ __forceinline__ uint16_t bf16_bits(float x) {
    __nv_bfloat16 v = __float2bfloat16_rn(x);
    return *reinterpret_cast<uint16_t *>(&v);
}
__device__ __forceinline__ void split1(float x, uint16_t &hi, uint16_t &lo) {
    hi = bf16_bits(x);
    lo = bf16_bits(x - __uint_as_float(static_cast<uint32_t>(hi) << 16));
}

// Swizzled bf16 tile of C columns (C = 64 or 128): 16-byte chunk c of row r is
// stored at chunk c ^ (r & 7), so ldmatrix's eight row reads hit distinct
// banks. Returns the element offset.
template <int C>
__device__ __forceinline__ int swz(int r, int c) {
    return r * C + ((((c >> 3) ^ (r & 7))) << 3) + (c & 7);
}

// ---------------------------------------------------------------------------
// Shared-memory map (bytes), for head dim D
// ---------------------------------------------------------------------------

template <int D>
struct Smem {
    static constexpr int FS = D + 8;                       // fp32 tile row stride (conflict-free float2)
    static constexpr int AS = BT + 4;                      // fp32 64x64 tile row stride
    static constexpr int kRawQ = 0;                        // bf16 [64][D]   q of the chunk
    static constexpr int kRawK = kRawQ + BT * D * 2;       // bf16 [64][D]   k
    static constexpr int kRawG = kRawK + BT * D * 2;       // fp32 [64][D]   g (bf16 a for the raw gate)
    static constexpr int kRawEnd = kRawG + BT * D * 4;
    // A' and T (fp32 [64][AS]) alias the raw region once X/Y/Z are built.
    static constexpr int kAp = 0;
    static constexpr int kT = kAp + BT * AS * 4;
    static constexpr int kRawBytes = (kRawEnd > kT + BT * AS * 4) ? kRawEnd : kT + BT * AS * 4;
    static constexpr int kV = kRawBytes;                   // bf16 [64][D] swizzled, v of the chunk
    static constexpr int kX = kV + BT * D * 2;             // fp32 [64][FS]  X, then W hi/lo
    static constexpr int kY = kX + BT * FS * 4;            // fp32 [64][FS]  Y, then QG hi/lo
    static constexpr int kZ = kY + BT * FS * 4;            // fp32 [64][FS]  Z, then KD hi/lo
    static constexpr int kTBh = kZ + BT * FS * 4;          // bf16 [64][64] swizzled
    static constexpr int kTBl = kTBh + BT * BT * 2;
    static constexpr int kAQh = kTBl + BT * BT * 2;
    static constexpr int kAQl = kAQh + BT * BT * 2;
    static constexpr int kVec = kAQl + BT * BT * 2;        // fp32 vectors below
    // vector offsets in floats from kVec
    static constexpr int vRq = 0, vRk = 64, vBeta = 128;
    static constexpr int vM = 192;                         // [4][D] anchors m_I
    static constexpr int vEm = vM + 4 * D;                 // [4][D] e^{m_I}
    static constexpr int vF = vEm + 4 * D;                 // [6][D] e^{m_I - m_J}, J < I
    static constexpr int vTot = vF;                        // [4][D] cumsum partial totals (before vF)
    static constexpr int vEglm = vF + 6 * D;               // [4][D] e^{gl - m_J}
    static constexpr int vEgl = vEglm + 4 * D;             // [D]    e^{gl}
    static constexpr int vGl = vEgl + D;                   // [D]    gl = gc of the last row
    static constexpr int vGtr = vGl + D;                   // [D]    gc of the tracked row
    static constexpr int vEtr = vGtr + D;                  // [D]    e^{gtr}
    static constexpr int vEnd = vEtr + D;
    static constexpr int kBytes = kVec + vEnd * 4;
    static_assert(kBytes <= 232448, "chunk kernel shared memory exceeds the 227 KiB per-CTA limit");
};

// Block pair index p -> (I, J), J <= I, in the order (0,0) (1,0) (1,1) (2,0) ...
__device__ __forceinline__ void pair_ij(int p, int &I, int &J) {
    I = (p >= 6) ? 3 : (p >= 3) ? 2 : (p >= 1) ? 1 : 0;
    J = p - I * (I + 1) / 2;
}
// Factor slot of an off-diagonal pair (J < I) in the vF table.
__device__ __forceinline__ int fslot(int I, int J) { return I * (I - 1) / 2 + J; }

// ldmatrix lane addresses (element offsets into a swizzled tile of C columns).
// A fragment (16x16) of a row-major [m][k] tile at (m0, k0).
template <int C>
__device__ __forceinline__ int lda_a(int lane, int m0, int k0) {
    return swz<C>(m0 + (lane & 15), k0 + ((lane >> 4) << 3));
}
// Two n-tiles of B fragments (16 k x 16 n) from a [n][k] tile at (n0, k0).
template <int C>
__device__ __forceinline__ int lda_b_nk(int lane, int n0, int k0) {
    const int q = lane >> 3, r = lane & 7;
    return swz<C>(n0 + r + ((q >> 1) << 3), k0 + ((q & 1) << 3));
}
// Two n-tiles of B fragments from a [k][n] tile at (k0, n0), with .trans.
template <int C>
__device__ __forceinline__ int lda_b_kn(int lane, int k0, int n0) {
    const int q = lane >> 3, r = lane & 7;
    return swz<C>(k0 + r + ((q & 1) << 3), n0 + ((q >> 1) << 3));
}
// A fragment (16 m x 16 k) from a [k][m] tile at (m0, k0), with .trans.
template <int C>
__device__ __forceinline__ int lda_a_km(int lane, int m0, int k0) {
    const int q = lane >> 3, r = lane & 7;
    return swz<C>(k0 + r + ((q >> 1) << 3), m0 + ((q & 1) << 3));
}

// Ranks requests by length, longest first, so the longest chunk chains start
// first (one block; order[rank] = request).
__global__ void __launch_bounds__(1024) order_kernel(const KdaArgs p, int32_t *order) {
    __shared__ int32_t len[1024];
    const int n = p.num_req;
    for (int r = threadIdx.x; r < n; r += blockDim.x)
        len[r] = static_cast<int32_t>(load_index(p.cu_seqlens, p.index_bytes[1], r + 1) -
                                      load_index(p.cu_seqlens, p.index_bytes[1], r));
    __syncthreads();
    for (int r = threadIdx.x; r < n; r += blockDim.x) {
        int rank = 0;
        const int lr = len[r];
        for (int q = 0; q < n; ++q) rank += (len[q] > lr) || (len[q] == lr && q < r);
        order[rank] = r;
    }
}

template <int D, int MODE>
__global__ void __launch_bounds__(kThreads, 1) chunk_kernel(const KdaArgs p, const int32_t *order) {
    using L = Smem<D>;
    constexpr int KS = D / 16;              // k-steps over the key dim
    constexpr int NPART = kThreads / D;     // row parts of the column-per-thread mapping
    constexpr int RPT = BT / NPART;         // rows per thread in that mapping
    constexpr int SCAN_WARPS = D / 16;      // warps that own 16 value rows each
    constexpr int FS = L::FS, AS = L::AS;
    extern __shared__ __align__(128) unsigned char sm[];
    uint16_t *const rawQ = reinterpret_cast<uint16_t *>(sm + L::kRawQ);
    uint16_t *const rawK = reinterpret_cast<uint16_t *>(sm + L::kRawK);
    float *const rawG = reinterpret_cast<float *>(sm + L::kRawG);
    uint16_t *const rawA = reinterpret_cast<uint16_t *>(sm + L::kRawG);
    float *const Ap = reinterpret_cast<float *>(sm + L::kAp);
    float *const Tm = reinterpret_cast<float *>(sm + L::kT);
    uint16_t *const Vt = reinterpret_cast<uint16_t *>(sm + L::kV);
    float *const X = reinterpret_cast<float *>(sm + L::kX);
    float *const Y = reinterpret_cast<float *>(sm + L::kY);
    float *const Z = reinterpret_cast<float *>(sm + L::kZ);
    uint16_t *const Wh = reinterpret_cast<uint16_t *>(sm + L::kX);
    uint16_t *const Wl = Wh + BT * D;
    uint16_t *const QGh = reinterpret_cast<uint16_t *>(sm + L::kY);
    uint16_t *const QGl = QGh + BT * D;
    uint16_t *const KDh = reinterpret_cast<uint16_t *>(sm + L::kZ);
    uint16_t *const KDl = KDh + BT * D;
    uint16_t *const KRh = rawQ;             // tracked-prefix operand, in the raw region
    uint16_t *const KRl = rawK;
    uint16_t *const TBh = reinterpret_cast<uint16_t *>(sm + L::kTBh);
    uint16_t *const TBl = reinterpret_cast<uint16_t *>(sm + L::kTBl);
    uint16_t *const AQh = reinterpret_cast<uint16_t *>(sm + L::kAQh);
    uint16_t *const AQl = reinterpret_cast<uint16_t *>(sm + L::kAQl);
    float *const vec = reinterpret_cast<float *>(sm + L::kVec);
    const uint32_t s_base = smem_addr(sm);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int H = p.num_heads;
    const int rr = blockIdx.x / p.head_count;
    const int h = p.head_begin + blockIdx.x % p.head_count;
    const int req = order != nullptr ? order[rr] : rr;

    const int64_t bos = load_index(p.cu_seqlens, p.index_bytes[1], req);
    const int64_t eos = load_index(p.cu_seqlens, p.index_bytes[1], req + 1);
    const int64_t slot = load_index(p.indices, p.index_bytes[0], req);
    if (bos < 0 || eos < bos || eos > p.num_tokens) {
        if (tid == 0) report(p.status, KDA_DEVICE_ERR_BAD_SEQLENS);
        return;
    }
    if (slot < 0 || slot >= p.num_slots) {
        if (tid == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
        return;
    }
    int64_t tslot = 0, tlen = -1;
    if (p.track_indices != nullptr) {
        tslot = load_index(p.track_indices, p.index_bytes[2], req);
        if (tslot < 0 || tslot >= p.num_slots) {
            if (tid == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
            return;
        }
        if (tslot > 0) tlen = load_index(p.track_lens, p.index_bytes[3], req);
    }
    const int nchunks = static_cast<int>((eos - bos + BT - 1) / BT);
    const int64_t s0 = p.state_stride[0], s1 = p.state_stride[1], sk = p.state_stride[2], sv = p.state_stride[3];

    // Column-per-thread mapping of the elementwise passes.
    const int kc = tid % D, pt = tid / D;
    float dtb = 0.f, expA = 0.f;
    if constexpr (MODE == KDA_GATE_RAW) {
        dtb = __ldg(p.dt_bias + h * D + kc);
        expA = expf(__ldg(p.A_log + h));
    }

    auto issue_qkg = [&](int c) {
        const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
        const int n = static_cast<int>((eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT)));
        constexpr int CPR = D / 8;
        for (int e = tid; e < BT * CPR; e += kThreads) {
            const int i = e / CPR, cc = e % CPR;
            const bool ok = i < n;
            const int64_t off = (ok ? ((t0 + i) * H + h) * D : 0) + cc * 8;
            cp_async16(rawQ + i * D + cc * 8, static_cast<const uint16_t *>(p.q) + off, ok);
            cp_async16(rawK + i * D + cc * 8, static_cast<const uint16_t *>(p.k) + off, ok);
            if constexpr (MODE == KDA_GATE_RAW)
                cp_async16(rawA + i * D + cc * 8, static_cast<const uint16_t *>(p.a) + off, ok);
        }
        if constexpr (MODE == KDA_GATE_LOG) {
            constexpr int CPG = D / 4;
            for (int e = tid; e < BT * CPG; e += kThreads) {
                const int i = e / CPG, cc = e % CPG;
                const bool ok = i < n;
                const int64_t off = (ok ? ((t0 + i) * H + h) * D : 0) + cc * 4;
                cp_async16(rawG + i * D + cc * 4, p.g + off, ok);
            }
        }
    };
    auto issue_v = [&](int c) {
        const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
        const int n = static_cast<int>((eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT)));
        constexpr int CPR = D / 8;
        for (int e = tid; e < BT * CPR; e += kThreads) {
            const int i = e / CPR, cc = e % CPR;
            const bool ok = i < n;
            const int64_t off = (ok ? ((t0 + i) * H + h) * D : 0) + cc * 8;
            cp_async16(Vt + swz<D>(i, cc * 8), static_cast<const uint16_t *>(p.v) + off, ok);
        }
    };
    float bnext = 0.f;   // beta (or raw b) of row `tid` of the next chunk
    auto load_beta = [&](int c) {
        const int64_t tt = bos + static_cast<int64_t>(c) * BT + tid;
        if (tid < BT && tt < eos) {
            if constexpr (MODE == KDA_GATE_RAW)
                bnext = bf16_to_f(p.b, tt * H + h);
            else
                bnext = __ldg(p.beta + tt * H + h);
        }
    };

    // ---- state S^T in registers: warp w < SCAN_WARPS owns value rows
    // [16w, 16w + 16); fragment S[nt] covers key columns [8nt, 8nt + 8). ----
    const bool scan_warp = warp < SCAN_WARPS;
    const int vr = warp * 16 + g;                      // rows vr, vr + 8
    float S[D / 8][4];
    {
        const float *hs = p.state + slot * s0 + h * s1;
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
            const int k = nt * 8 + 2 * t4;
            const bool ld = scan_warp && slot > 0;
            S[nt][0] = ld ? hs[vr * sv + k * sk] : 0.f;
            S[nt][1] = ld ? hs[vr * sv + (k + 1) * sk] : 0.f;
            S[nt][2] = ld ? hs[(vr + 8) * sv + k * sk] : 0.f;
            S[nt][3] = ld ? hs[(vr + 8) * sv + (k + 1) * sk] : 0.f;
        }
    }
    auto store_state = [&](float *hs) {
#pragma unroll
        for (int nt = 0; nt < D / 8; ++nt) {
            const int k = nt * 8 + 2 * t4;
            hs[vr * sv + k * sk] = S[nt][0];
            hs[vr * sv + (k + 1) * sk] = S[nt][1];
            hs[(vr + 8) * sv + k * sk] = S[nt][2];
            hs[(vr + 8) * sv + (k + 1) * sk] = S[nt][3];
        }
    };
    if (scan_warp && tslot > 0 && tlen == 0) store_state(p.state + tslot * s0 + h * s1);

    if (nchunks > 0) {
        issue_qkg(0);
        issue_v(0);
        cp_async_commit();
        load_beta(0);
    }

    for (int c = 0; c < nchunks; ++c) {
        const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
        const int n = static_cast<int>((eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT)));
        const int64_t rtrack = tlen - static_cast<int64_t>(c) * BT;
        const bool track_here = tslot > 0 && rtrack > 0 && rtrack <= BT;
        const bool has_next = c + 1 < nchunks;
        cp_async_wait_all();
        __syncthreads();

        // ---- P1: beta, row norms (scale folded into q), gate cumsum ----
        if (tid < BT) {
            float bt = 0.f;
            if (tid < n) {
                if constexpr (MODE == KDA_GATE_RAW)
                    bt = sigmoidf_(bnext);
                else
                    bt = bnext;
            }
            vec[L::vBeta + tid] = bt;
        }
        {
            const int grp = tid >> 4, l16 = tid & 15;
            constexpr int EPL = D / 16;             // elements per lane of a row
#pragma unroll
            for (int it = 0; it < 8; ++it) {
                const int rowid = grp + 16 * it;   // 0..63 q rows, 64..127 k rows
                const int row = rowid & 63;
                const uint16_t *src = (rowid >= 64 ? rawK : rawQ) + row * D + l16 * EPL;
                float ss = 0.f;
#pragma unroll
                for (int e = 0; e < EPL; ++e) {
                    const float x = __uint_as_float(static_cast<uint32_t>(src[e]) << 16);
                    ss = fmaf(x, x, ss);
                }
                ss += __shfl_xor_sync(0xffffffffu, ss, 8);
                ss += __shfl_xor_sync(0xffffffffu, ss, 4);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                if (l16 == 0) {
                    const float inv = 1.0f / sqrtf(ss + kNormEps);
                    if (rowid >= 64)
                        vec[L::vRk + row] = inv;
                    else
                        vec[L::vRq + row] = p.scale * inv;
                }
            }
        }
        float gcr[RPT];
        const int trow = track_here ? static_cast<int>(rtrack) - 1 : -1;   // gc row of the checkpoint
        float gtr = 0.f;
        {
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = pt * RPT + i;
                float gv;
                if constexpr (MODE == KDA_GATE_RAW) {
                    const float av = __uint_as_float(static_cast<uint32_t>(rawA[row * D + kc]) << 16);
                    gv = row < n ? p.lower_bound * sigmoidf_(expA * (av + dtb)) : 0.f;
                } else {
                    gv = rawG[row * D + kc];
                }
                acc += gv;
                gcr[i] = acc;
                gtr = (row == trow) ? acc : gtr;
            }
            if (pt < NPART - 1) vec[L::vTot + pt * D + kc] = acc;
        }
        __syncthreads();
        {
            float off = 0.f;
            for (int q = 0; q < pt; ++q) off += vec[L::vTot + q * D + kc];
#pragma unroll
            for (int i = 0; i < RPT; ++i) gcr[i] += off;
            gtr += off;
        }
        __syncthreads();   // vTot is read; vF (its alias) is written below

        // ---- P2a: anchors, last/tracked gate rows, X/Y/Z ----
#pragma unroll
        for (int lb = 0; lb < RPT / 16; ++lb) vec[L::vM + (pt * RPT / 16 + lb) * D + kc] = gcr[lb * 16 + 8];
        if (pt == NPART - 1) vec[L::vGl + kc] = gcr[RPT - 1];
        if (trow >= 0 && trow / RPT == pt) vec[L::vGtr + kc] = gtr;
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int row = pt * RPT + i;
            const float m = gcr[(i / 16) * 16 + 8];
            const float x = gcr[i] - m;
            const float E = expf(x), Ei = expf(-x);
            const float kn = __uint_as_float(static_cast<uint32_t>(rawK[row * D + kc]) << 16) * vec[L::vRk + row];
            const float qn = __uint_as_float(static_cast<uint32_t>(rawQ[row * D + kc]) << 16) * vec[L::vRq + row];
            X[row * FS + kc] = kn * E;
            Y[row * FS + kc] = qn * E;
            Z[row * FS + kc] = kn * Ei;
        }
        __syncthreads();

        // ---- P2b: per-(block, column) factors ----
        for (int e = tid; e < 16 * D; e += kThreads) {
            const int r = e / D, k = e % D;
            if (r < 4) {
                vec[L::vEm + r * D + k] = expf(vec[L::vM + r * D + k]);
            } else if (r < 10) {
                const int s = r - 4;
                const int I = (s < 1) ? 1 : (s < 3) ? 2 : 3;
                const int J = s - I * (I - 1) / 2;
                vec[L::vF + s * D + k] = expf(vec[L::vM + I * D + k] - vec[L::vM + J * D + k]);
            } else if (r < 14) {
                const int J = r - 10;
                vec[L::vEglm + J * D + k] = expf(vec[L::vGl + k] - vec[L::vM + J * D + k]);
            } else if (r == 14) {
                vec[L::vEgl + k] = expf(vec[L::vGl + k]);
            } else {
                vec[L::vEtr + k] = track_here ? expf(vec[L::vGtr + k]) : 0.f;
            }
        }
        __syncthreads();

        // ---- P3: A' and Aqk, one 16x16 block pair per warp pass ----
        for (int pidx = warp; pidx < 10; pidx += kWarps) {
            int I, J;
            pair_ij(pidx, I, J);
            const float *F = (J < I) ? vec + L::vF + fslot(I, J) * D : nullptr;
            float akk[2][4] = {}, aqk[2][4] = {};
            const int ra = 16 * I + g, rb = ra + 8;
#pragma unroll 2
            for (int ks = 0; ks < KS; ++ks) {
                const int c0 = ks * 16 + 2 * t4;
                float2 f0 = make_float2(1.f, 1.f), f1 = make_float2(1.f, 1.f);
                if (F != nullptr) {
                    f0 = *reinterpret_cast<const float2 *>(F + c0);
                    f1 = *reinterpret_cast<const float2 *>(F + c0 + 8);
                }
                uint32_t xh[4], xl[4], yh[4], yl[4];
                {
                    const float2 a0 = *reinterpret_cast<const float2 *>(X + ra * FS + c0);
                    const float2 a1 = *reinterpret_cast<const float2 *>(X + rb * FS + c0);
                    const float2 a2 = *reinterpret_cast<const float2 *>(X + ra * FS + c0 + 8);
                    const float2 a3 = *reinterpret_cast<const float2 *>(X + rb * FS + c0 + 8);
                    split2(a0.x * f0.x, a0.y * f0.y, xh[0], xl[0]);
                    split2(a1.x * f0.x, a1.y * f0.y, xh[1], xl[1]);
                    split2(a2.x * f1.x, a2.y * f1.y, xh[2], xl[2]);
                    split2(a3.x * f1.x, a3.y * f1.y, xh[3], xl[3]);
                }
                {
                    const float2 a0 = *reinterpret_cast<const float2 *>(Y + ra * FS + c0);
                    const float2 a1 = *reinterpret_cast<const float2 *>(Y + rb * FS + c0);
                    const float2 a2 = *reinterpret_cast<const float2 *>(Y + ra * FS + c0 + 8);
                    const float2 a3 = *reinterpret_cast<const float2 *>(Y + rb * FS + c0 + 8);
                    split2(a0.x * f0.x, a0.y * f0.y, yh[0], yl[0]);
                    split2(a1.x * f0.x, a1.y * f0.y, yh[1], yl[1]);
                    split2(a2.x * f1.x, a2.y * f1.y, yh[2], yl[2]);
                    split2(a3.x * f1.x, a3.y * f1.y, yh[3], yl[3]);
                }
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const int j = 16 * J + 8 * nt + g;
                    const float2 z0 = *reinterpret_cast<const float2 *>(Z + j * FS + c0);
                    const float2 z1 = *reinterpret_cast<const float2 *>(Z + j * FS + c0 + 8);
                    uint32_t bh0, bl0, bh1, bl1;
                    split2(z0.x, z0.y, bh0, bl0);
                    split2(z1.x, z1.y, bh1, bl1);
                    mma3(akk[nt], xh, xl, bh0, bh1, bl0, bl1);
                    mma3(aqk[nt], yh, yl, bh0, bh1, bl0, bl1);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
                for (int hf = 0; hf < 2; ++hf) {
                    const int i = 16 * I + g + 8 * hf;
                    const int j0 = 16 * J + 8 * nt + 2 * t4;
                    const float bi = vec[L::vBeta + i];
                    const float a0 = (j0 < i) ? akk[nt][2 * hf] * bi : 0.f;
                    const float a1 = (j0 + 1 < i) ? akk[nt][2 * hf + 1] * bi : 0.f;
                    *reinterpret_cast<float2 *>(Ap + i * AS + j0) = make_float2(a0, a1);
                    const float q0 = (j0 <= i) ? aqk[nt][2 * hf] : 0.f;
                    const float q1 = (j0 + 1 <= i) ? aqk[nt][2 * hf + 1] : 0.f;
                    uint32_t qh, ql;
                    split2(q0, q1, qh, ql);
                    *reinterpret_cast<uint32_t *>(AQh + swz<BT>(i, j0)) = qh;
                    *reinterpret_cast<uint32_t *>(AQl + swz<BT>(i, j0)) = ql;
                }
            }
        }
        __syncthreads();

        // ---- P4: T = (I + A')^-1, blocked forward substitution in fp32 ----
        if (warp < 4 && lane < 16) {
            const int I = warp, j = lane;
            float col[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                float acc = (i == j) ? 1.f : 0.f;
                const float *arow = Ap + (16 * I + i) * AS + 16 * I;
#pragma unroll
                for (int m = 0; m < i; ++m)
                    if (m >= j) acc -= arow[m] * col[m];
                col[i] = (i >= j) ? acc : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) Tm[(16 * I + i) * AS + 16 * I + j] = col[i];
        }
        __syncthreads();
        {
            const int i = tid >> 4, j = tid & 15;
#pragma unroll
            for (int d = 1; d <= 3; ++d) {
                float res[3];
#pragma unroll
                for (int q = 0; q < 4 - d; ++q) {
                    const int I = d + q, J = q;
                    float acc = 0.f;
                    for (int M = J; M < I; ++M) {
                        const float *arow = Ap + (16 * I + i) * AS + 16 * M;
                        const float *tcol = Tm + (16 * M) * AS + 16 * J + j;
#pragma unroll
                        for (int m = 0; m < 16; ++m) acc = fmaf(arow[m], tcol[m * AS], acc);
                    }
                    res[q] = acc;
                }
#pragma unroll
                for (int q = 0; q < 4 - d; ++q) Tm[(16 * (d + q) + i) * AS + 16 * q + j] = res[q];
                __syncthreads();
#pragma unroll
                for (int q = 0; q < 4 - d; ++q) {
                    const int I = d + q, J = q;
                    const float *trow = Tm + (16 * I + i) * AS + 16 * I;
                    const float *pcol = Tm + (16 * I) * AS + 16 * J + j;
                    float acc = 0.f;
#pragma unroll
                    for (int m = 0; m < 16; ++m) acc = fmaf(trow[m], pcol[m * AS], acc);
                    res[q] = -acc;
                }
                __syncthreads();
#pragma unroll
                for (int q = 0; q < 4 - d; ++q) Tm[(16 * (d + q) + i) * AS + 16 * q + j] = res[q];
                __syncthreads();
            }
        }

        // ---- P5: TB = T diag(beta), lower triangle, split into hi/lo ----
        for (int e = tid; e < BT * (BT / 2); e += kThreads) {
            const int j = e / (BT / 2), jc = (e % (BT / 2)) * 2;
            const float x0 = (jc <= j) ? Tm[j * AS + jc] * vec[L::vBeta + jc] : 0.f;
            const float x1 = (jc + 1 <= j) ? Tm[j * AS + jc + 1] * vec[L::vBeta + jc + 1] : 0.f;
            uint32_t hi, lo;
            split2(x0, x1, hi, lo);
            *reinterpret_cast<uint32_t *>(TBh + swz<BT>(j, jc)) = hi;
            *reinterpret_cast<uint32_t *>(TBl + swz<BT>(j, jc)) = lo;
        }
        __syncthreads();

        // ---- P6: the raw region is free: fetch the next chunk's q/k/g ----
        if (has_next && !track_here) {
            issue_qkg(c + 1);
            cp_async_commit();
            load_beta(c + 1);
        }

        // ---- P7: W = TB (kn e^{gc}); warp w owns key columns [16w, 16w+16) ----
        float wacc[4][2][4] = {};
        if (warp < D / 16) {
            uint32_t kbh[4][2][2], kbl[4][2][2];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    const int kcol = 16 * warp + 8 * nt + g;
                    const int jr = 16 * ks + 2 * t4;
                    const float e = vec[L::vEm + ks * D + kcol];
                    split2(X[jr * FS + kcol] * e, X[(jr + 1) * FS + kcol] * e, kbh[ks][nt][0], kbl[ks][nt][0]);
                    split2(X[(jr + 8) * FS + kcol] * e, X[(jr + 9) * FS + kcol] * e, kbh[ks][nt][1],
                           kbl[ks][nt][1]);
                }
            }
#pragma unroll
            for (int mt = 0; mt < 4; ++mt) {
#pragma unroll
                for (int ks = 0; ks <= mt; ++ks) {
                    uint32_t ah[4], al[4];
                    ldsm_x4(ah, s_base + L::kTBh + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
                    ldsm_x4(al, s_base + L::kTBl + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
                        mma3(wacc[mt][nt], ah, al, kbh[ks][nt][0], kbh[ks][nt][1], kbl[ks][nt][0], kbl[ks][nt][1]);
                }
            }
        }
        __syncthreads();   // X fully consumed: W replaces it
        if (warp < D / 16) {
#pragma unroll
            for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int hf = 0; hf < 2; ++hf) {
                        const int j = 16 * mt + g + 8 * hf;
                        const int kcol = 16 * warp + 8 * nt + 2 * t4;
                        uint32_t hi, lo;
                        split2(wacc[mt][nt][2 * hf], wacc[mt][nt][2 * hf + 1], hi, lo);
                        *reinterpret_cast<uint32_t *>(Wh + swz<D>(j, kcol)) = hi;
                        *reinterpret_cast<uint32_t *>(Wl + swz<D>(j, kcol)) = lo;
                    }
        }

        // ---- P8: QG = Y e^{m_I}, KD = Z e^{gl - m_J}, tracked K_r, in place ----
        {
            uint32_t stage[RPT];
            const float etr_k = track_here ? vec[L::vGtr + kc] : 0.f;
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = pt * RPT + i;
                const int I = row / 16;
                uint16_t hi, lo;
                split1(Y[row * FS + kc] * vec[L::vEm + I * D + kc], hi, lo);
                stage[i] = static_cast<uint32_t>(hi) | (static_cast<uint32_t>(lo) << 16);
                if (track_here) {
                    const float kr = (row < rtrack) ? Z[row * FS + kc] * expf(etr_k - vec[L::vM + I * D + kc]) : 0.f;
                    split1(kr, hi, lo);
                    KRh[swz<D>(row, kc)] = hi;
                    KRl[swz<D>(row, kc)] = lo;
                }
            }
            __syncthreads();
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = pt * RPT + i;
                QGh[swz<D>(row, kc)] = static_cast<uint16_t>(stage[i] & 0xffffu);
                QGl[swz<D>(row, kc)] = static_cast<uint16_t>(stage[i] >> 16);
            }
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = pt * RPT + i;
                uint16_t hi, lo;
                split1(Z[row * FS + kc] * vec[L::vEglm + (row / 16) * D + kc], hi, lo);
                stage[i] = static_cast<uint32_t>(hi) | (static_cast<uint32_t>(lo) << 16);
            }
            __syncthreads();
#pragma unroll
            for (int i = 0; i < RPT; ++i) {
                const int row = pt * RPT + i;
                KDh[swz<D>(row, kc)] = static_cast<uint16_t>(stage[i] & 0xffffu);
                KDl[swz<D>(row, kc)] = static_cast<uint16_t>(stage[i] >> 16);
            }
        }
        __syncthreads();

        // ---- P9: the scan, each warp on its 16 value rows ----
        float U[8][4] = {};   // u^T, then -v'^T  (value rows x 64 chunk rows)
        if (scan_warp) {
#pragma unroll
            for (int np = 0; np < 4; ++np) {
#pragma unroll
                for (int ks = 0; ks <= np; ++ks) {
                    uint32_t av[4], bh[4], bl[4];
                    ldsm_x4_t(av, s_base + L::kV + 2 * lda_a_km<D>(lane, warp * 16, 16 * ks));
                    ldsm_x4(bh, s_base + L::kTBh + 2 * lda_b_nk<BT>(lane, 16 * np, 16 * ks));
                    ldsm_x4(bl, s_base + L::kTBl + 2 * lda_b_nk<BT>(lane, 16 * np, 16 * ks));
                    mma16816(U[2 * np], av, bl[0], bl[1]);
                    mma16816(U[2 * np], av, bh[0], bh[1]);
                    mma16816(U[2 * np + 1], av, bl[2], bl[3]);
                    mma16816(U[2 * np + 1], av, bh[2], bh[3]);
                }
            }
#pragma unroll
            for (int nt = 0; nt < 8; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) U[nt][e] = -U[nt][e];
        }
        __syncthreads();   // the v tile is consumed: fetch the next one
        if (has_next && !track_here) {
            issue_v(c + 1);
            cp_async_commit();
        }
        if (scan_warp) {
            float O[8][4] = {};
#pragma unroll
            for (int ks = 0; ks < KS; ++ks) {
                uint32_t sh[4], sl[4];
                split2(S[2 * ks][0], S[2 * ks][1], sh[0], sl[0]);
                split2(S[2 * ks][2], S[2 * ks][3], sh[1], sl[1]);
                split2(S[2 * ks + 1][0], S[2 * ks + 1][1], sh[2], sl[2]);
                split2(S[2 * ks + 1][2], S[2 * ks + 1][3], sh[3], sl[3]);
#pragma unroll
                for (int np = 0; np < 4; ++np) {
                    uint32_t bh[4], bl[4];
                    ldsm_x4(bh, s_base + L::kX + 2 * lda_b_nk<D>(lane, 16 * np, 16 * ks));
                    ldsm_x4(bl, s_base + L::kX + 2 * BT * D + 2 * lda_b_nk<D>(lane, 16 * np, 16 * ks));
                    mma3(U[2 * np], sh, sl, bh[0], bh[1], bl[0], bl[1]);
                    mma3(U[2 * np + 1], sh, sl, bh[2], bh[3], bl[2], bl[3]);
                    ldsm_x4(bh, s_base + L::kY + 2 * lda_b_nk<D>(lane, 16 * np, 16 * ks));
                    ldsm_x4(bl, s_base + L::kY + 2 * BT * D + 2 * lda_b_nk<D>(lane, 16 * np, 16 * ks));
                    mma3(O[2 * np], sh, sl, bh[0], bh[1], bl[0], bl[1]);
                    mma3(O[2 * np + 1], sh, sl, bh[2], bh[3], bl[2], bl[3]);
                }
            }
            // v'^T fragments (A operand over the chunk rows j), from -U.
            uint32_t vh[4][4], vl[4][4];
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                split2(-U[2 * ks][0], -U[2 * ks][1], vh[ks][0], vl[ks][0]);
                split2(-U[2 * ks][2], -U[2 * ks][3], vh[ks][1], vl[ks][1]);
                split2(-U[2 * ks + 1][0], -U[2 * ks + 1][1], vh[ks][2], vl[ks][2]);
                split2(-U[2 * ks + 1][2], -U[2 * ks + 1][3], vh[ks][3], vl[ks][3]);
            }
#pragma unroll
            for (int np = 0; np < 4; ++np) {
#pragma unroll
                for (int ks = 0; ks <= np; ++ks) {
                    uint32_t bh[4], bl[4];
                    ldsm_x4(bh, s_base + L::kAQh + 2 * lda_b_nk<BT>(lane, 16 * np, 16 * ks));
                    ldsm_x4(bl, s_base + L::kAQl + 2 * lda_b_nk<BT>(lane, 16 * np, 16 * ks));
                    mma3(O[2 * np], vh[ks], vl[ks], bh[0], bh[1], bl[0], bl[1]);
                    mma3(O[2 * np + 1], vh[ks], vl[ks], bh[2], bh[3], bl[2], bl[3]);
                }
            }
            // Output rows of this chunk: o[t0 + i][h][v].
#pragma unroll
            for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const int i = 8 * nt + 2 * t4 + (e & 1);
                    const int v = vr + ((e & 2) ? 8 : 0);
                    if (i < n) {
                        const int64_t oi = ((t0 + i) * H + h) * D + v;
                        if (p.out_fp32)
                            static_cast<float *>(p.out)[oi] = O[nt][e];
                        else
                            static_cast<__nv_bfloat16 *>(p.out)[oi] = __float2bfloat16_rn(O[nt][e]);
                    }
                }
            }
            // Tracked prefix: S_r^T = S^T e^{gc_{r-1}} + v'^T K_r, stored, S unchanged.
            if (track_here) {
                float *hs = p.state + tslot * s0 + h * s1;
#pragma unroll
                for (int half = 0; half < 2; ++half) {
                    float R[D / 16][4];
#pragma unroll
                    for (int q = 0; q < D / 16; ++q) {
                        const int nt = half * (D / 16) + q;
                        const int k = nt * 8 + 2 * t4;
                        const float e0 = vec[L::vEtr + k], e1 = vec[L::vEtr + k + 1];
                        R[q][0] = S[nt][0] * e0;
                        R[q][1] = S[nt][1] * e1;
                        R[q][2] = S[nt][2] * e0;
                        R[q][3] = S[nt][3] * e1;
                    }
#pragma unroll
                    for (int np = 0; np < D / 32; ++np) {
#pragma unroll
                        for (int ks = 0; ks < 4; ++ks) {
                            uint32_t bh[4], bl[4];
                            const int n0 = half * (D / 2) + 16 * np;
                            ldsm_x4_t(bh, s_base + L::kRawQ + 2 * lda_b_kn<D>(lane, 16 * ks, n0));
                            ldsm_x4_t(bl, s_base + L::kRawK + 2 * lda_b_kn<D>(lane, 16 * ks, n0));
                            mma3(R[2 * np], vh[ks], vl[ks], bh[0], bh[1], bl[0], bl[1]);
                            mma3(R[2 * np + 1], vh[ks], vl[ks], bh[2], bh[3], bl[2], bl[3]);
                        }
                    }
#pragma unroll
                    for (int q = 0; q < D / 16; ++q) {
                        const int k = (half * (D / 16) + q) * 8 + 2 * t4;
                        hs[vr * sv + k * sk] = R[q][0];
                        hs[vr * sv + (k + 1) * sk] = R[q][1];
                        hs[(vr + 8) * sv + k * sk] = R[q][2];
                        hs[(vr + 8) * sv + (k + 1) * sk] = R[q][3];
                    }
                }
            }
            // State update: S^T = S^T e^{gl} + v'^T KD.
#pragma unroll
            for (int nt = 0; nt < D / 8; ++nt) {
                const int k = nt * 8 + 2 * t4;
                const float e0 = vec[L::vEgl + k], e1 = vec[L::vEgl + k + 1];
                S[nt][0] *= e0;
                S[nt][1] *= e1;
                S[nt][2] *= e0;
                S[nt][3] *= e1;
            }
#pragma unroll
            for (int np = 0; np < D / 16; ++np) {
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t bh[4], bl[4];
                    ldsm_x4_t(bh, s_base + L::kZ + 2 * lda_b_kn<D>(lane, 16 * ks, 16 * np));
                    ldsm_x4_t(bl, s_base + L::kZ + 2 * BT * D + 2 * lda_b_kn<D>(lane, 16 * ks, 16 * np));
                    mma3(S[2 * np], vh[ks], vl[ks], bh[0], bh[1], bl[0], bl[1]);
                    mma3(S[2 * np + 1], vh[ks], vl[ks], bh[2], bh[3], bl[2], bl[3]);
                }
            }
        }
        if (track_here && has_next) {
            __syncthreads();   // K_r (raw region) is consumed
            issue_qkg(c + 1);
            issue_v(c + 1);
            cp_async_commit();
            load_beta(c + 1);
        }
    }
    cp_async_wait_all();
    if (scan_warp && slot > 0) store_state(p.state + slot * s0 + h * s1);
}

}  // namespace chunk

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static bool chunk_aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static size_t order_bytes(int32_t num_req) {
    return (static_cast<size_t>(num_req > 0 ? num_req : 1) * sizeof(int32_t) + 255) / 256 * 256;
}

template <int D, int MODE>
static int launch_chunk(const KdaArgs *a, int32_t *order, cudaStream_t st) {
    using L = chunk::Smem<D>;
    static bool opted[64];
    int dev = 0;
    cudaGetDevice(&dev);
    dev = (dev >= 0 && dev < 64) ? dev : 0;
    if (!opted[dev]) {
        if (cudaFuncSetAttribute(chunk::chunk_kernel<D, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 L::kBytes) != cudaSuccess)
            return KDA_ERR_LAUNCH;
        opted[dev] = true;
    }
    if (order != nullptr) chunk::order_kernel<<<1, 1024, 0, st>>>(*a, order);
    const int64_t grid = static_cast<int64_t>(a->num_req) * a->head_count;
    chunk::chunk_kernel<D, MODE><<<static_cast<unsigned>(grid), chunk::kThreads, L::kBytes, st>>>(*a, order);
    return KDA_OK;
}

}  // namespace kda

extern "C" size_t kda_chunk_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads,
                                            int32_t head_dim) {
    (void)num_tokens;
    (void)num_heads;
    (void)head_dim;
    return (num_req > 0 && num_req <= 1024) ? kda::order_bytes(num_req) : 0;
}

extern "C" int kda_chunk_launch(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream) {
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->intermediate != nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_PREPARED) return KDA_ERR_UNSUPPORTED;
    if (args->head_dim != 64 && args->head_dim != 128) return KDA_ERR_UNSUPPORTED;
    if (args->num_req < 0 || args->num_tokens < 0 || args->num_heads <= 0 || args->head_begin < 0 ||
        args->head_count < 0 || args->head_begin + args->head_count > args->num_heads)
        return KDA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 4; ++i)
        if (args->index_bytes[i] != 4 && args->index_bytes[i] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (args->num_req == 0 || args->head_count == 0) return KDA_OK;
    if (args->state == nullptr || args->num_slots <= 0 || args->indices == nullptr || args->cu_seqlens == nullptr ||
        args->out == nullptr || args->q == nullptr || args->k == nullptr || args->v == nullptr)
        return KDA_ERR_INVALID_ARGUMENT;
    if ((args->track_indices == nullptr) != (args->track_lens == nullptr)) return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_RAW &&
        (args->a == nullptr || args->b == nullptr || args->A_log == nullptr || args->dt_bias == nullptr))
        return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_LOG && (args->g == nullptr || args->beta == nullptr))
        return KDA_ERR_INVALID_ARGUMENT;
    // cp.async moves 16-byte pieces of q/k/v/a/g rows.
    const void *rows[] = {args->q, args->k, args->v, args->gate_mode == KDA_GATE_RAW ? args->a : args->g};
    for (const void *ptr : rows)
        if (!kda::chunk_aligned16(ptr)) return KDA_ERR_ALIGNMENT;
    const size_t need = kda_chunk_workspace_bytes(args->num_req, args->num_tokens, args->num_heads, args->head_dim);
    int32_t *order = nullptr;
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes < need) return KDA_ERR_WORKSPACE;
        if ((reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) return KDA_ERR_ALIGNMENT;
        order = static_cast<int32_t *>(workspace);
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int rc;
    if (args->head_dim == 128)
        rc = args->gate_mode == KDA_GATE_RAW ? kda::launch_chunk<128, KDA_GATE_RAW>(args, order, st)
                                             : kda::launch_chunk<128, KDA_GATE_LOG>(args, order, st);
    else
        rc = args->gate_mode == KDA_GATE_RAW ? kda::launch_chunk<64, KDA_GATE_RAW>(args, order, st)
                                             : kda::launch_chunk<64, KDA_GATE_LOG>(args, order, st);
    if (rc != KDA_OK) return rc;
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}

// ---------------------------------------------------------------------------
// Allocation-free variant of kda_chunk_launch
//
// Some callers cannot hand this library a workspace: a host that reserved
// (almost) all device memory for its own pools before the first call, or a
// runtime bound through a foreign-function layer that has no device allocator
// at all. For them the only scratch this operator needs -- the longest-first
// request order, one int32 per request -- lives in a fixed array inside the
// library instead. It holds KDA_CHUNK_STATIC_MAX_REQUESTS entries (4 KiB);
// every GPU that loads the library carries one copy until the process exits.
// ---------------------------------------------------------------------------

static __device__ __align__(256) int32_t g_chunk_order_scratch[KDA_CHUNK_STATIC_MAX_REQUESTS];

namespace kda {

// Device address of the scratch array on the current device. Looked up once
// per device (with that device current) and cached; the array's host-side
// name is only a handle and must never reach a kernel.
static int chunk_static_scratch(int32_t **out) {
    static std::mutex mu;
    static int32_t *addr[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return KDA_ERR_LAUNCH;
    std::lock_guard<std::mutex> lk(mu);
    if (addr[dev] == nullptr) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_chunk_order_scratch) != cudaSuccess || ptr == nullptr)
            return KDA_ERR_LAUNCH;
        addr[dev] = static_cast<int32_t *>(ptr);
    }
    *out = addr[dev];
    return KDA_OK;
}

}  // namespace kda

extern "C" int kda_chunk_launch_no_alloc(const KdaArgs *args, void *stream) {
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->num_req > KDA_CHUNK_STATIC_MAX_REQUESTS) return KDA_ERR_TOO_LARGE;
    int32_t *scratch = nullptr;
    if (args->num_req > 0) {
        const int rc = kda::chunk_static_scratch(&scratch);
        if (rc != KDA_OK) return rc;
    }
    // The order kernel rewrites entries [0, num_req) on every call, so the
    // array needs no clearing; only concurrent calls would interfere.
    return kda_chunk_launch(args, scratch, sizeof(int32_t) * KDA_CHUNK_STATIC_MAX_REQUESTS, stream);
}
