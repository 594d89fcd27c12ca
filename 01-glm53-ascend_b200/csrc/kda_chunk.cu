// Chunk-64 WY/UT prefill of the GLM KDA operator on sm_100a, behind
// kda_chunk_launch / kda_chunk_workspace_bytes / kda_chunk_launch_no_alloc.
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
//   * one CTA per (sequence, head), the whole chunk loop in one CTA; requests
//     are visited longest-first (a one-block prologue kernel writes the order
//     into the workspace). 16 compute warps plus one producer warp whose
//     single thread issues every TMA load and every tcgen05 product, in the
//     order mbarrier signals from the compute warps allow, so no compute warp
//     blocks on a tensor-core issue queue.
//   * every tensor-core product splits each inexact fp32 operand into hi + lo
//     bf16 and issues three products (hi.hi + hi.lo + lo.hi): plain bf16
//     operands miss the output bar (5e-3 of the output RMS) by 3-13x on these
//     inputs, the split form lands at ~2e-4.
//   * the exponent range is handled with 16-row blocks anchored at their
//     midpoint row, the anchor rounded to a multiple of ln 2:
//     X = kn e^{gc - m_I}, Y = qn e^{gc - m_I} and Z = kn e^{m_I - gc} stay
//     within e^{+-(8|g| + ln2/2)} and are split into bf16 hi/lo once; a block
//     pair (I, J) is X_I (e^{m_I - m_J}) Z_J^T where the factor is an exact
//     power of two <= 1, applied to Z's bf16 fragments without rounding, and
//     QG = Y e^{m_I}, kn e^{gc} = X e^{m_I} likewise (fp32 exp overflows at
//     e^88.7; the reference rebases per 32 rows for the same reason,
//     kda_varlen_chunk.h:24-29).
//   * intra-chunk products (A blocks, inverse levels, W) run on mma.sync with
//     ldmatrix fragments; the state scan runs on the 5th-gen tensor core: the
//     state S^T (value rows x key columns, the pool's own [V][K] order) lives
//     in tensor memory as a 128-lane fp32 accumulator, its bf16 hi/lo split is
//     stored back to tensor memory and used as the A operand, and the
//     intra-chunk results (W, QG, KD, TB, Aqk) are B operands in 128-byte
//     swizzled shared-memory tiles. Conversions of tensor memory (state split,
//     v', output) are spread over compute warps that the intra-chunk phases
//     leave idle.
//   * the next chunk's q/k/g (and v) tiles are fetched by TMA (one tensor
//     map each, the v tile written in the 128-byte swizzle the tensor core
//     reads) while this chunk runs, each as soon as its shared-memory region
//     is dead (q, k and g after the inverse, v after u = TB v);
//     output tiles leave by TMA stores.
//   * any sequence length: a partial last chunk is zero-filled (k = q = v =
//     g = beta = 0), which leaves the state and the real rows unchanged.
//     Requests of 1..16 tokens go to the token recurrence instead (launched
//     first by kda_chunk_launch), where a token costs one step, not a chunk.
//   * every mbarrier wait is bounded; tensor memory is freed on every path.

#include "kda_common.cuh"

#include <cuda.h>
#include <cstdlib>
#include <cstring>
#include <algorithm>
#include <mutex>

namespace kda {
namespace chunk {

constexpr int BT = 64;
constexpr int kThreads = 512;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

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

__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r[0]), "=r"(r[1])
                 : "r"(addr));
}

// 2^x on the special-function unit (relative error ~2^-22, flushes denormals).
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}
// bf16x2 product; exact when one factor is a power of two and nothing leaves
// the normal range (an underflow flushes a vanishing term to zero).
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
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
// tcgen05 (5th-gen tensor core) primitives: tensor-memory allocation,
// single-thread MMA issue, commit to an mbarrier, warp loads/stores of tensor
// memory, and the shared-memory / instruction descriptors.
// ---------------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}
// Named barrier `id` over `count` threads (whole warps).
__device__ __forceinline__ void nbar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes -> visible to the tensor core (async proxy).
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] x B[smem desc]
__device__ __forceinline__ void umma_ss(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// D[tmem] (+)= A[tmem] x B[smem desc]
__device__ __forceinline__ void umma_ts(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d),
        "r"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
// All previously issued MMAs of this thread arrive on `bar` when complete.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
                 : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
                 : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};"
                 :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
                 : "memory");
}
// N consecutive fp32 columns of this warp's 32 lanes (N = 16 or 32).
template <int N>
__device__ __forceinline__ void tmem_ld(uint32_t taddr, uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
}
template <int N>
__device__ __forceinline__ void tmem_st(uint32_t taddr, const uint32_t (&r)[N]) {
    if constexpr (N == 32) tmem_st32(taddr, r);
    else if constexpr (N == 16) tmem_st16(taddr, r);
    else tmem_st8(taddr, r);
}

// Tiled TMA store of a 3-D box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_addr(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
// Linear bulk copy shared -> global (16-byte aligned ends, bytes % 16 == 0).
__device__ __forceinline__ void bulk_s2g(void *gdst, const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// This thread's committed bulk stores have finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Tiled TMA load of a 3-D box (x = key/value column, y = head, z = token)
// into shared memory, completing on `bar`. No multicast.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// L2 prefetch of the same 3-D box (no shared-memory destination, no barrier).
// L2 prefetch of a linear range (16-byte aligned, bytes % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void *src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(z)
                 : "memory");
}
// Tensor maps of one launch: q, k, the gate (g fp32, or a bf16 for the raw
// gate) as [T][H][D] boxes of 64 tokens x D, v as 64-token x 64-column
// boxes written with the 128-byte swizzle the tensor core reads, and the bf16
// output as 64-token x D boxes (stores of whole chunks).
struct TmaMaps {
    CUtensorMap q, k, g, v, o;
};

// Shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm_100
// version bit. Byte offsets: lbo = leading (MN-block) stride, sbo = 8-row
// group stride.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | (2ull << 61);
}
// No-swizzle K-major descriptor (layout type 0): core matrices of 8 rows x 16
// bytes stored contiguously; lbo = byte stride between core matrices along K,
// sbo = between core matrices along M (or N).
__device__ __forceinline__ uint64_t sdesc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}
// The descriptor of (s_base + off) from the descriptor of s_base with the same
// lbo/sbo: the start-address field holds address >> 4 in bits 0-13, and a
// CTA's shared-memory addresses stay below 2^18 bytes, so adding off >> 4
// never carries out of it. With `off` a compile-time constant this is one
// integer add per tensor-core instruction the producer thread issues.
__device__ __forceinline__ uint64_t sdesc_add(uint64_t base, uint32_t off) { return base + (off >> 4); }
// `x` made opaque where it is computed, so the compiler keeps the producer's
// descriptor bases inside the producer's loop instead of hoisting them (and
// every constant offset from them) into registers live across the kernel.
__device__ __forceinline__ uint64_t opaque64(uint64_t x) {
    asm volatile("" : "+l"(x));
    return x;
}

// Instruction descriptor: fp32 accumulate, bf16 A and B, dense.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N, bool a_mn, bool b_mn, bool b_neg) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((b_neg ? 1u : 0u) << 14) | ((a_mn ? 1u : 0u) << 15) |
           ((b_mn ? 1u : 0u) << 16) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Tensor-memory column map (512 columns allocated; lane = value row).
constexpr uint32_t kColS = 0;      // fp32 S^T, D columns
constexpr uint32_t kColSH = 128;   // bf16x2 hi of S^T, D/2 columns
constexpr uint32_t kColSL = 192;   // bf16x2 lo of S^T
constexpr uint32_t kColTR = 128;   // fp32 tracked-prefix state, D columns (reuses SH/SL once consumed)
constexpr uint32_t kColNU = 256;   // fp32 -v'^T, 64 columns
constexpr uint32_t kColO = 320;    // fp32 o^T, 64 columns
constexpr uint32_t kColVH = 384;   // bf16x2 hi of v'^T, 32 columns
constexpr uint32_t kColVL = 416;   // bf16x2 lo of v'^T
constexpr uint32_t kTmemCols = 512;

// ---------------------------------------------------------------------------
// Shared-memory map (bytes from a 1024-byte aligned base), for head dim D
// ---------------------------------------------------------------------------

__host__ __device__ constexpr int r1k(int x) { return (x + 1023) / 1024 * 1024; }

// bf16 tiles of 64 rows use 64-column blocks in the canonical 128-byte swizzle
// atom (8 rows x 128 B, 16-byte chunk c of row r at c ^ (r & 7)): element
// (r, c) of a 64 x C tile sits at (c / 64) * 4096 + swz<64>(r, c % 64).
__device__ __forceinline__ int f64(int r, int c) { return ((c >> 6) << 12) + swz<64>(r, c & 63); }

template <int D>
struct Smem {
    static constexpr int AS = BT + 4;                      // fp32 64x64 tile row stride
    static constexpr int kRawQ = 0;                        // bf16 [64][D]   q of the chunk (plain rows)
    static constexpr int kRawK = kRawQ + BT * D * 2;       // bf16 [64][D]   k
    static constexpr int kRawG = kRawK + BT * D * 2;       // fp32 [64][D]   g (bf16 a for the raw gate),
                                                           //                then x = gc - m (in place)
    static constexpr int kRawEnd = kRawG + BT * D * 4;
    // A' and T (fp32 [64][AS]) alias the raw region once X/Y/Z are built;
    // the tracked-prefix operand K_r (hi at kRawQ, lo at kRawK) as well.
    static constexpr int kAp = 0;
    static constexpr int kT = kAp + BT * AS * 4;
    static constexpr int PS = 20;                          // row stride of the P scratch blocks
    static constexpr int kP = kT + BT * AS * 4;            // fp32 [4][16][PS] inverse partial products
    // bf16 [64][D] o tile of the previous chunk, staged for its TMA store
    // while A', T and P occupy the front of the raw region.
    static constexpr int kOst = r1k(kP + 4 * 16 * PS * 4);
    static constexpr int kOstEnd = kOst + BT * D * 2;
    static constexpr int kV = r1k(kRawEnd > kOstEnd ? kRawEnd : kOstEnd);   // bf16 f64 tile [j][v]
    // bf16 hi/lo f64 tiles (hi at the base, lo BT*D*2 bytes later):
    static constexpr int kX = r1k(kV + BT * D * 2);        // X, then W
    static constexpr int kY = kX + BT * D * 4;             // Y, then QG (in place)
    static constexpr int kZ = kY + BT * D * 4;             // Z, then KD (in place)
    static constexpr int kTBh = kZ + BT * D * 4;           // bf16 [64][64] swizzled
    static constexpr int kTBl = kTBh + BT * BT * 2;
    static constexpr int kAQh = kTBl + BT * BT * 2;
    static constexpr int kAQl = kAQh + BT * BT * 2;
    static constexpr int kBar = kAQl + BT * BT * 2;        // 9 mbarriers + tensor-memory base slot
    static constexpr int kVec = kBar + 128;                // vectors below
    // vector offsets in 4-byte words from kVec; per (16-row block I, column k)
    // tables are [4][D]
    static constexpr int vRq = 0, vRk = 64, vBeta = 128;
    static constexpr int vM = 192;                         // [4][D] anchors m_I (multiples of ln 2)
    static constexpr int vTot = vM + 4 * D;                // [4][D] cumsum block totals
    static constexpr int vS = vTot + 4 * D;                // bf16 [4][D] 2^{m_I / ln 2} = e^{m_I}
    static constexpr int vFb = vS + 2 * D;                 // bf16 [6][D] e^{m_I - m_J}, J < I
    static constexpr int vEglm = vFb + 3 * D;              // [4][D] e^{gl - m_J}
    static constexpr int vEtrm = vEglm + 4 * D;            // [4][D] e^{gtr - m_J} (tracked chunk)
    static constexpr int vEgl = vEtrm + 4 * D;             // [D]    e^{gl}
    static constexpr int vGl = vEgl + D;                   // [D]    gl = gc of the last row
    static constexpr int vGtr = vGl + D;                   // [D]    gc of the tracked row
    static constexpr int vEtr = vGtr + D;                  // [D]    e^{gtr}
    static constexpr int vEnd = vEtr + D;
    static constexpr int kBytes = kVec + vEnd * 4;
    static constexpr int kAlloc = kBytes + 1024;           // room to align the base to 1024 B
    static_assert(kAlloc <= 232448, "chunk kernel shared memory exceeds the 227 KiB per-CTA limit");
};

// Split path (long sequences, few (sequence, head) chains): the prep kernel
// stores each chunk-head's scan operands as one record, in the shared-memory
// layout the scan kernel reads, so every part is a single bulk copy.
template <int D>
struct Rec {
    static constexpr int kW = 0;                       // bf16 hi/lo f64 tiles [64][D] (W)
    static constexpr int kQG = kW + BT * D * 4;         // QG
    static constexpr int kKD = kQG + BT * D * 4;        // KD
    // -u^T = -(TB v)^T, fp32, float (t, v) at ((t / 4) * D + v) * 4 + t % 4: a
    // compute warp reads its 16 tokens of value row v as four 16-byte pieces,
    // eight consecutive rows per 128 bytes.
    static constexpr int kU = kKD + BT * D * 4;
    static constexpr int kAQ = kU + BT * D * 4;         // Aqk (bf16 hi/lo [64][64] swizzled)
    static constexpr int kEgl = kAQ + BT * BT * 4;      // fp32 [D] e^{gl}
    static constexpr int kBytes = r1k(kEgl + D * 4);
    // per (request, head): the tracked-prefix operand and e^{gtr}
    static constexpr int tKR = 0;                       // bf16 hi/lo f64 [64][D]
    static constexpr int tEtr = BT * D * 4;             // fp32 [D]
    static constexpr int tBytes = r1k(tEtr + D * 4);
};

// Split path: what the scan leaves for the output kernel per chunk-head --
// the chunk-start state S^T as bf16 hi/lo, value rows x key columns, in
// groups of 8 columns: element (r, c) of an R-row tile at (c / 8 * R + r) * 8
// + c % 8. A warp's 32 rows of one group are one 512-byte store, and the 8
// rows an ldmatrix reads are 128 contiguous bytes. (The output kernel keeps
// v' in the same layout, [D][64] (value, token).)
template <int D>
struct ScanOut {
    static constexpr int kSH = 0;                       // [D][D]  (value, key)
    static constexpr int kSL = kSH + D * D * 2;
    static constexpr int kBytes = r1k(kSL + D * D * 2);
};
template <int R>
__device__ __forceinline__ int fr(int r, int c) { return ((c >> 3) * R + r) * 8 + (c & 7); }

// Split path, segmented scan. The state recurrence of one (sequence, head) is
// affine, S_{c+1} = A_c S_c + B_c (A_c = diag(e^{gl}) - KD^T W, B_c = KD^T u),
// so a long sequence is cut into P segments of about L chunks that scan side
// by side: segment 0 from the true initial state, and segments 1..P-2 twice,
// once from zero (their B) and once from the identity with u = 0 (their A);
// both chains also leave their state at the segment's midpoint, and the last
// segment gets the same two chains over its first half only. A combine step
// then chains S_start[i+1] = A_i S_start[i] + B_i, and every segment i >= 1
// rescans as two halves side by side: the first from S_start[i], the second
// from S_mid[i] = A_mid,i S_start[i] + B_mid,i, one product in its prologue.
// The rescan stores the splits the output kernel reads. Two segments gain
// nothing, so a sequence has 1 or >= 3.
//
// The plan (int32 words in the workspace, written by plan_kernel):
//   [0] state-slot capacity, [1] first-pass task count, [2] rescan task
//   count, [3] task capacity, then per request: segments P_r, segment length
//   L_r (chunks), first state slot; then the first-pass and rescan task lists.
// A task is req | kind << 10 | half << 12 | segment << 13 (half: a chain over
// the first half of a segment only, or the second half of a rescan).
enum : int { kTaskTrue = 0, kTaskZero = 1, kTaskIdent = 2 };
constexpr int kMinSegChunks = 8;
struct PlanView {
    int32_t *w;
    int R, cap;
    __host__ __device__ PlanView(int32_t *words, int num_req, int task_cap) : w(words), R(num_req), cap(task_cap) {}
    __device__ int32_t *segs() const { return w + 4; }
    __device__ int32_t *seglen() const { return w + 4 + R; }
    __device__ int32_t *sbase() const { return w + 4 + 2 * R; }
    __device__ int32_t *tasks(int phase) const { return w + 4 + 3 * R + phase * cap; }
    __host__ __device__ static size_t words(int num_req, int task_cap) {
        return 4 + 3 * static_cast<size_t>(num_req) + 2 * static_cast<size_t>(task_cap);
    }
};
__device__ __forceinline__ int32_t task_word(int req, int kind, int seg, int half = 0) {
    return req | (kind << 10) | (half << 12) | (seg << 13);
}
// State-slot kinds per (request, segment >= 1, head).
enum : int { kSlotStart = 0, kSlotB = 1, kSlotA = 2, kSlotBmid = 3, kSlotAmid = 4, kSlotKinds = 5 };
// State exchange layout of one D x D fp32 state S^T (value row v, key column
// k): float at ((k / 4) D + v) * 4 + k % 4, so a warp's 32 rows of one float4
// column are 512 contiguous bytes. Slot `slot` of kind `which` (0 start
// states, 1 segment B, 2 segment A) for head hl:
template <int D>
__device__ __forceinline__ float *state_slot(float *states, int cap, int heads, int which, int slot, int hl) {
    return states + ((static_cast<int64_t>(which) * cap + slot) * heads + hl) * (D * D);
}

// Exclusive prefix sum over a 1024-thread block (one value per thread); the
// total lands in `total`. Every thread of the block must call it.
__device__ int block_scan(int x, int32_t *tmp, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int v = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) tmp[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int w = tmp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += y;
        }
        tmp[lane] = w;
    }
    __syncthreads();
    const int before = (warp > 0 ? tmp[warp - 1] : 0) + v - x;
    total = tmp[31];
    __syncthreads();
    return before;
}
__device__ int block_max(int x, int32_t *tmp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) x = max(x, __shfl_xor_sync(0xffffffffu, x, o));
    if (lane == 0) tmp[warp] = x;
    __syncthreads();
    int m = tmp[0];
    for (int i = 1; i < 32; ++i) m = max(m, tmp[i]);
    __syncthreads();
    return m;
}

// Block pair (I, J), J <= I, of P3's warp w: warps 0..9 take (1,0) (2,0)
// (0,0) (1,1) (2,1) (3,0) (2,2) (3,3) (3,1) (3,2). The four diagonal blocks,
// whose warps also solve T_II, sit on sub-partitions 2 and 3 (w % 4), which
// hold two product warps each against three on sub-partitions 0 and 1.
__device__ __forceinline__ void pair_ij(int w, int &I, int &J) {
    // 4 bits per warp: I in bits 0-1, J in bits 2-3
    constexpr uint64_t kPairs = 0x1ull | (0x2ull << 4) | (0x0ull << 8) | (0x5ull << 12) | (0x6ull << 16) |
                                (0x3ull << 20) | (0xAull << 24) | (0xFull << 28) | (0x7ull << 32) |
                                (0xBull << 36);
    const int v = static_cast<int>((kPairs >> (4 * w)) & 0xFu);
    I = v & 3;
    J = v >> 2;
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

// The same lane addresses for the 64-row f64 tiles (64-column blocks; a
// 16-column span never crosses a block).
__device__ __forceinline__ int fa_a(int lane, int m0, int k0) {
    return f64(m0 + (lane & 15), k0 + ((lane >> 4) << 3));
}
__device__ __forceinline__ int fb_nk(int lane, int n0, int k0) {
    const int q = lane >> 3, r = lane & 7;
    return f64(n0 + r + ((q >> 1) << 3), k0 + ((q & 1) << 3));
}
// B fragments (16 k x 8 n) from a [k][n] f64 tile at (k0, n0), with .trans (x2).
__device__ __forceinline__ int fb_kn8(int lane, int k0, int n0) {
    return f64(k0 + (lane & 7) + (((lane >> 3) & 1) << 3), n0);
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

template <int D, int MODE, bool PREP>
__global__ void __launch_bounds__(kThreads + 32, 1)
    chunk_kernel(const KdaArgs p, const int32_t *order, const __grid_constant__ TmaMaps maps, uint8_t *rec,
                 uint8_t *trec, const int32_t *cbase, int32_t skip_hi) {
    using L = Smem<D>;
    constexpr int KS = D / 16;              // k-steps over the key dim
    constexpr int ELEM = 4 * D;             // threads of the column-per-thread passes
    constexpr int RPT = 16;                 // rows per thread in those passes (one 16-row block)
    constexpr int AS = L::AS;
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    uint16_t *const rawQ = reinterpret_cast<uint16_t *>(sm + L::kRawQ);
    uint16_t *const rawK = reinterpret_cast<uint16_t *>(sm + L::kRawK);
    float *const rawG = reinterpret_cast<float *>(sm + L::kRawG);
    uint16_t *const rawA = reinterpret_cast<uint16_t *>(sm + L::kRawG);
    float *const Ap = reinterpret_cast<float *>(sm + L::kAp);
    float *const Tm = reinterpret_cast<float *>(sm + L::kT);
    float *const Pp = reinterpret_cast<float *>(sm + L::kP);
    uint16_t *const Vt = reinterpret_cast<uint16_t *>(sm + L::kV);
    float *const xg = reinterpret_cast<float *>(sm + L::kRawG);   // x = gc - m, in place of the gate
    uint16_t *const Xh = reinterpret_cast<uint16_t *>(sm + L::kX);
    uint16_t *const Xl = Xh + BT * D;
    uint16_t *const Yh = reinterpret_cast<uint16_t *>(sm + L::kY);
    uint16_t *const Yl = Yh + BT * D;
    uint16_t *const Zh = reinterpret_cast<uint16_t *>(sm + L::kZ);
    uint16_t *const Zl = Zh + BT * D;
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
    // o tile staging: in the W region at the end of a tracked chunk and after
    // the last chunk, in the raw region during the next chunk's inverse
    __nv_bfloat16 *const OstX = reinterpret_cast<__nv_bfloat16 *>(sm + L::kX);
    __nv_bfloat16 *const OstR = reinterpret_cast<__nv_bfloat16 *>(sm + L::kOst);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(sm + L::kBar);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(sm + L::kBar + 64);
    // CTA-wide give-up word of the bounded waits (between the tensor-memory
    // slot and sig_a)
    volatile int32_t *const abort_w = reinterpret_cast<volatile int32_t *>(sm + L::kBar + 68);
    float *const vec = reinterpret_cast<float *>(sm + L::kVec);
    const uint32_t s_base = smem_addr(sm);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int H = p.num_heads;
    const int h = p.head_begin + blockIdx.x % p.head_count;
    int req, cprep = 0;   // PREP: this CTA's request and chunk within it
    if constexpr (PREP) {
        // Chunk slot -> (request, chunk): cbase[r] = chunks of requests < r.
        const int sl = blockIdx.x / p.head_count;
        int r = 0;
        while (r < p.num_req && cbase[r + 1] <= sl) ++r;
        if (r >= p.num_req) return;   // past the batch's last chunk
        req = r;
        cprep = sl - cbase[r];
    } else {
        const int rr = blockIdx.x / p.head_count;
        req = order != nullptr ? order[rr] : rr;
    }

    const int64_t bos = load_index(p.cu_seqlens, p.index_bytes[1], req);
    const int64_t eos = load_index(p.cu_seqlens, p.index_bytes[1], req + 1);
    const int64_t slot = load_index(p.indices, p.index_bytes[0], req);
    // Requests of 1..skip_hi tokens went to the token recurrence of the same
    // launch (kda_chunk_launch's fused path): nothing to do here.
    if (eos - bos >= 1 && eos - bos <= skip_hi) return;
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

    // Column-per-thread mapping of the elementwise passes: column kc, rows
    // [16 pt, 16 pt + 16) -- one anchor block per thread.
    const bool elem = tid < ELEM;
    const int kc = tid % D, pt = tid / D;
    float dtb = 0.f, expA = 0.f;
    if constexpr (MODE == KDA_GATE_RAW) {
        if (elem) dtb = __ldg(p.dt_bias + h * D + kc);
        expA = expf(__ldg(p.A_log + h));
    }

    auto chunk_rows = [&](int c) {
        const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
        return static_cast<int>(eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT));
    };
    // Tiles of chunk c by TMA, issued by thread 0, all completing on bars[2]:
    // q, k and the gate at once, v (the first scan product's A operand) either
    // with them or once the previous chunk's product has consumed its tile.
    constexpr uint32_t kTileBytes =
        BT * D * 2 * 3 + BT * D * ((MODE == KDA_GATE_RAW) ? 2 : 4);
    auto issue_v = [&](int c) {
        const int t0c = static_cast<int>(bos + static_cast<int64_t>(c) * BT);
#pragma unroll
        for (int blk = 0; blk < D / 64; ++blk) tma_load_3d(Vt + blk * 4096, &maps.v, 64 * blk, h, t0c, &bars[2]);
    };
    // Untracked chunks split the copy: q once A' (the front of the raw region)
    // is dead, k and the gate once the rest of the region is free.
    auto issue_q = [&](int c) {
        const int t0c = static_cast<int>(bos + static_cast<int64_t>(c) * BT);
        mbar_arrive_expect_tx(&bars[2], kTileBytes);
        tma_load_3d(rawQ, &maps.q, 0, h, t0c, &bars[2]);
    };
    auto issue_kg = [&](int c) {
        const int t0c = static_cast<int>(bos + static_cast<int64_t>(c) * BT);
        tma_load_3d(rawK, &maps.k, 0, h, t0c, &bars[2]);
        tma_load_3d(rawG, &maps.g, 0, h, t0c, &bars[2]);
    };
    auto issue_tiles = [&](int c, bool with_v, bool expect_v = true) {
        const int t0c = static_cast<int>(bos + static_cast<int64_t>(c) * BT);
        mbar_arrive_expect_tx(&bars[2], expect_v ? kTileBytes : kTileBytes - BT * D * 2);
        tma_load_3d(rawQ, &maps.q, 0, h, t0c, &bars[2]);
        tma_load_3d(rawK, &maps.k, 0, h, t0c, &bars[2]);
        tma_load_3d(rawG, &maps.g, 0, h, t0c, &bars[2]);
        if (with_v) issue_v(c);
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

    // ---- tensor memory, mbarriers ----
    // bars: 0 = W S done (v' ready), 1 = state update done, 2 = chunk tiles
    // landed, 3 = o^T done, 4 = u product done (v tile free). sig: consumer ->
    // producer, 0 = TB/QG/S-split ready, 1 = W/KD ready, 2 = v' hi/lo ready;
    // sig_a = A' read for the last time (P4 done). (The tensor-memory slot
    // sits between bars[7] and sig_a.)
    uint64_t *const sig = bars + 5;
    uint64_t *const sig_a = bars + 9;
    if (!PREP && warp == 0) tmem_alloc(tmem_slot, kTmemCols);
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) mbar_init(&bars[i], 1);
        mbar_init(sig_a, 1);
        *abort_w = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = PREP ? 0u : *tmem_slot;
    // Tensor-memory slices: warp w reaches lanes [32 (w % 4), +32) (value
    // rows) and takes column slice w / 4 of every conversion.
    const int q4 = warp & 3, cs = warp >> 2;
    const int srow = 32 * q4 + lane;                 // value row of this thread
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    constexpr int SC = D / 4;                        // state columns per slice

    if (PREP && warp == kThreads / 32) {
        // Prep: this CTA's one chunk of q, k, the gate and v; then an L2
        // prefetch of the tiles of the CTA one wave later (block + SM count),
        // which is dispatched about when a CTA of this wave retires.
        if (lane == 0) {
            issue_tiles(cprep, true);
            uint32_t nsm;
            asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
            const int64_t nb = static_cast<int64_t>(blockIdx.x) + nsm;
            if (nb < static_cast<int64_t>(gridDim.x)) {
                const int sl2 = static_cast<int>(nb / p.head_count);
                const int h2 = p.head_begin + static_cast<int>(nb % p.head_count);
                int r2 = 0;
                while (r2 < p.num_req && cbase[r2 + 1] <= sl2) ++r2;
                if (r2 < p.num_req) {
                    const int t2 = static_cast<int>(load_index(p.cu_seqlens, p.index_bytes[1], r2) +
                                                    static_cast<int64_t>(sl2 - cbase[r2]) * BT);
                    tma_prefetch_3d(&maps.q, 0, h2, t2);
                    tma_prefetch_3d(&maps.k, 0, h2, t2);
                    tma_prefetch_3d(&maps.g, 0, h2, t2);
#pragma unroll
                    for (int blk = 0; blk < D / 64; ++blk) tma_prefetch_3d(&maps.v, 64 * blk, h2, t2);
                }
            }
        }
    } else if (warp == kThreads / 32) {
        // ===== producer warp: one thread issues every tensor-core product and
        // every TMA load, in the order the consumers' signals allow =====
        if (lane == 0 && nchunks > 0) {
            constexpr uint32_t id_v = idesc_bf16(128, 64, true, false, true);      // -(v^T TB^T)
            constexpr uint32_t id_n64 = idesc_bf16(128, 64, false, false, false);
            constexpr uint32_t id_kd = idesc_bf16(128, D, false, true, false);
            auto pwait = [&](uint64_t *b, uint32_t ph) {
                if (!mbar_wait(b, ph, p.status, abort_w)) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            };
            issue_tiles(0, true);
            for (int c = 0; c < nchunks; ++c) {
                const uint64_t d16 = opaque64(sdesc(s_base, 16, 1024)), d8k = opaque64(sdesc(s_base, 8192, 1024));
                const uint32_t ph = static_cast<uint32_t>(c & 1);
                const int64_t rt = tlen - static_cast<int64_t>(c) * BT;
                const bool trk = tslot > 0 && rt > 0 && rt <= BT;
                const bool nxt = c + 1 < nchunks;
                pwait(sig_a, ph);
                if (nxt && !trk) issue_q(c + 1);    // A' is dead: q's part of the raw region is free
                pwait(&sig[0], ph);
                tc_fence_after();
                if (nxt && !trk) issue_kg(c + 1);   // the raw region is free
                // NU = -u^T = -(TB v)^T (needs neither S nor v')
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint64_t a = sdesc_add(d8k, L::kV + kk * 2048);
                    umma_ss(tmem + kColNU, a, sdesc_add(d16, L::kTBh + kk * 32), id_v, kk > 0 ? 1u : 0u);
                    umma_ss(tmem + kColNU, a, sdesc_add(d16, L::kTBl + kk * 32), id_v, 1u);
                }
                umma_commit(&bars[4]);
                if (nxt && !trk) {
                    pwait(&bars[4], ph);   // the v tile is consumed
                    issue_v(c + 1);
                }
                pwait(&sig[1], ph);
                tc_fence_after();
                // NU += (W S)^T  ->  -v'^T
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t ah = tmem + kColSH + 8 * kk, al = tmem + kColSL + 8 * kk;
                    const uint32_t off = (kk >> 2) * 8192 + (kk & 3) * 32;
                    const uint64_t wh = sdesc_add(d16, L::kX + off);
                    const uint64_t wl = sdesc_add(d16, L::kX + BT * D * 2 + off);
                    umma_ts(tmem + kColNU, al, wh, id_n64, 1u);
                    umma_ts(tmem + kColNU, ah, wl, id_n64, 1u);
                    umma_ts(tmem + kColNU, ah, wh, id_n64, 1u);
                }
                if (!trk) umma_commit(&bars[0]);
                // o^T = (QG S)^T, while the consumers convert v' (on a tracked
                // chunk before bars[0]: the conversion reuses the S hi/lo columns)
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t ah = tmem + kColSH + 8 * kk, al = tmem + kColSL + 8 * kk;
                    const uint32_t off = (kk >> 2) * 8192 + (kk & 3) * 32;
                    const uint64_t qh = sdesc_add(d16, L::kY + off);
                    const uint64_t ql = sdesc_add(d16, L::kY + BT * D * 2 + off);
                    umma_ts(tmem + kColO, al, qh, id_n64, kk > 0 ? 1u : 0u);
                    umma_ts(tmem + kColO, ah, ql, id_n64, 1u);
                    umma_ts(tmem + kColO, ah, qh, id_n64, 1u);
                }
                if (trk) umma_commit(&bars[0]);
                pwait(&sig[2], ph);
                tc_fence_after();
                // S^T += v'^T KD (and the tracked prefix), then o^T += v'^T Aqk^T.
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t ah = tmem + kColVH + 8 * kk, al = tmem + kColVL + 8 * kk;
                    const uint64_t dh = sdesc_add(d8k, L::kZ + kk * 2048);
                    const uint64_t dl = sdesc_add(d8k, L::kZ + BT * D * 2 + kk * 2048);
                    umma_ts(tmem + kColS, al, dh, id_kd, 1u);
                    umma_ts(tmem + kColS, ah, dl, id_kd, 1u);
                    umma_ts(tmem + kColS, ah, dh, id_kd, 1u);
                    if (trk) {
                        const uint64_t rh = sdesc_add(d8k, L::kRawQ + kk * 2048);
                        const uint64_t rl = sdesc_add(d8k, L::kRawK + kk * 2048);
                        umma_ts(tmem + kColTR, al, rh, id_kd, 1u);
                        umma_ts(tmem + kColTR, ah, rl, id_kd, 1u);
                        umma_ts(tmem + kColTR, ah, rh, id_kd, 1u);
                    }
                }
                umma_commit(&bars[1]);
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t ah = tmem + kColVH + 8 * kk, al = tmem + kColVL + 8 * kk;
                    const uint64_t qh = sdesc_add(d16, L::kAQh + kk * 32);
                    const uint64_t ql = sdesc_add(d16, L::kAQl + kk * 32);
                    umma_ts(tmem + kColO, al, qh, id_n64, 1u);
                    umma_ts(tmem + kColO, ah, ql, id_n64, 1u);
                    umma_ts(tmem + kColO, ah, qh, id_n64, 1u);
                }
                umma_commit(&bars[3]);
                if (nxt && trk) {
                    pwait(&bars[1], ph);   // K_r (raw region) and the v tile are consumed
                    issue_tiles(c + 1, true);
                }
            }
        }
    } else {
        // ===== consumer warps 0..15 =====
        auto cbar = [] { nbar(1, kThreads); };
        // o^T columns [c0, c0 + ncol) of this warp's lanes -> bf16 staging tile
        // (row-major [64][D]), or straight to `out` for fp32 verification output.
        auto o_cols = [&](__nv_bfloat16 *ost, int64_t ot0, int on, int c0, int ncol) {
            for (int cc = c0; cc < c0 + ncol; cc += 16) {
                uint32_t r[16];
                tmem_ld16(tq + kColO + cc, r);
                tmem_ld_wait();
                if (srow < D) {
                    if (p.out_fp32) {
                        float *o = static_cast<float *>(p.out) + (ot0 * H + h) * D + srow;
                        const int64_t row_stride = static_cast<int64_t>(H) * D;
#pragma unroll
                        for (int e = 0; e < 16; ++e)
                            if (cc + e < on) o[(cc + e) * row_stride] = __uint_as_float(r[e]);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e) ost[(cc + e) * D + srow] = __float2bfloat16_rn(__uint_as_float(r[e]));
                    }
                }
            }
        };
        // A staged o tile -> `out`: one TMA tile store for a whole chunk, row
        // copies for a partial one (rows past the sequence belong to the next).
        auto o_store = [&](const __nv_bfloat16 *ost, int64_t ot0, int on) {
            if (p.out_fp32) return;
            if (on == BT) {
                tma_store_3d(&maps.o, ost, 0, h, static_cast<int>(ot0));
            } else {
                __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + (ot0 * H + h) * D;
                for (int rw = 0; rw < on; ++rw)
                    bulk_s2g(o + static_cast<int64_t>(rw) * H * D, ost + rw * D, D * 2);
            }
            bulk_commit();
        };

        // Initial state S^T -> tensor memory (zero for slot 0 and the padding rows
        // of D = 64); a length-0 prefix checkpoint is the initial state.
        if (!PREP) {
            const float *hs = p.state + slot * s0 + h * s1;
            float *ts = p.state + tslot * s0 + h * s1;
            const bool row_ok = srow < D;
            uint32_t r[SC];
#pragma unroll
            for (int e = 0; e < SC; ++e) {
                const int k = SC * cs + e;
                const float x = (slot > 0 && row_ok) ? hs[srow * sv + k * sk] : 0.f;
                r[e] = __float_as_uint(x);
                if (row_ok && tslot > 0 && tlen == 0) ts[srow * sv + k * sk] = x;
            }
            tmem_st<SC>(tq + kColS + SC * cs, r);
            tmem_st_wait();
        }
        if (nchunks > 0) load_beta(cprep);
        // TB's and Aqk's strictly-upper 16x16 blocks are never computed but are
        // read by the full-width products: zero both tiles once (the chunks
        // rewrite only their lower blocks).
        for (int e = tid; e < 4 * BT * BT / 8; e += kThreads)
            reinterpret_cast<uint4 *>(TBh)[e] = make_uint4(0u, 0u, 0u, 0u);   // TBh, TBl, AQh, AQl are contiguous

        bool o_pending = false;   // the previous chunk's o^T waits in tensor memory
        bool ox_busy = false;     // thread 0: an o tile store still reads the W region
        int64_t o_t0 = 0;
        int o_n = 0;
        for (int c = cprep; c < (PREP ? cprep + 1 : nchunks); ++c) {
            const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
            const int n = chunk_rows(c);
            const int64_t rtrack = tlen - static_cast<int64_t>(c) * BT;
            const bool track_here = tslot > 0 && rtrack > 0 && rtrack <= BT;
            const bool has_next = !PREP && c + 1 < nchunks;
            if (!mbar_wait(&bars[2], static_cast<uint32_t>(PREP ? 0 : c & 1), p.status, abort_w) && tid == 0)
                report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            // A tracked chunk's o tile (thread 0's only store in flight) has
            // left the W region before P2 rewrites it.
            if (tid == 0 && ox_busy) {
                bulk_wait_read();
                ox_busy = false;
            }
            if (n < BT) {
                // The boxes cover 64 tokens; rows past this sequence's end hold the
                // next sequence (or TMA's zero fill past T): clear them.
                for (int e = n * (D / 8) + tid; e < BT * (D / 8); e += kThreads) {   // 8-element groups
                    reinterpret_cast<uint4 *>(rawQ)[e] = make_uint4(0u, 0u, 0u, 0u);
                    reinterpret_cast<uint4 *>(rawK)[e] = make_uint4(0u, 0u, 0u, 0u);
                    reinterpret_cast<uint4 *>(Vt)[((e / (D / 8)) * 8 + (e % 8)) + ((e % (D / 8)) / 8) * 512] =
                        make_uint4(0u, 0u, 0u, 0u);
                    if constexpr (MODE == KDA_GATE_RAW) {
                        reinterpret_cast<uint4 *>(rawA)[e] = make_uint4(0u, 0u, 0u, 0u);
                    } else {
                        reinterpret_cast<float4 *>(rawG)[2 * e] = make_float4(0.f, 0.f, 0.f, 0.f);
                        reinterpret_cast<float4 *>(rawG)[2 * e + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
                    }
                }
                fence_async_smem();
            }
            cbar();

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
                // Four threads per row of q (rows 0..63) or k (64..127); part p
                // reads the row's 16-byte groups 4i + p, with i mirrored on odd
                // rows so the two rows of a quarter-warp hit distinct banks.
                constexpr int GPT = D / 32;                       // groups per thread
                const int rowid = tid >> 2, part = tid & 3, row = rowid & 63;
                const uint4 *src = reinterpret_cast<const uint4 *>((rowid >= 64 ? rawK : rawQ) + row * D);
                float sa = 0.f, sb = 0.f;
    #pragma unroll
                for (int i = 0; i < GPT; ++i) {
                    const uint4 u = src[4 * (i ^ (row & 1)) + part];
                    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    #pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float lo = bf16_lo(w[e]), hi = bf16_hi(w[e]);
                        sa = fmaf(lo, lo, sa);
                        sb = fmaf(hi, hi, sb);
                    }
                }
                float ss = sa + sb;
                ss += __shfl_xor_sync(0xffffffffu, ss, 1);
                ss += __shfl_xor_sync(0xffffffffu, ss, 2);
                if (part == 0) {
                    const float inv = 1.0f / sqrtf(ss + kNormEps);
                    if (rowid >= 64)
                        vec[L::vRk + row] = inv;
                    else
                        vec[L::vRq + row] = p.scale * inv;
                }
            }
            float gcr[RPT];
            const int trow = track_here ? static_cast<int>(rtrack) - 1 : -1;   // gc row of the checkpoint
            float gtr = 0.f;
            if (elem) {
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
                vec[L::vTot + pt * D + kc] = acc;
            }
            cbar();   // block totals, norms, beta; every raw gate value has been read
            if (elem) {
                float off = 0.f;
    #pragma unroll
                for (int q = 0; q < 3; ++q)
                    if (q < pt) off += vec[L::vTot + q * D + kc];
    #pragma unroll
                for (int i = 0; i < RPT; ++i) gcr[i] += off;
                gtr += off;
                // Anchor of block pt: the midpoint row's gc rounded to a multiple of
                // ln 2, so every ratio of anchors is an exact power of two. Then
                // x = gc - m in place of the gate (|x| <= 8|g| + ln2/2).
                const float nI = rintf(gcr[8] * kLog2e);
                const float m = nI * kLn2;
                vec[L::vM + pt * D + kc] = m;
                reinterpret_cast<uint16_t *>(vec + L::vS)[pt * D + kc] =
                    nI >= -126.f ? static_cast<uint16_t>((static_cast<int>(nI) + 127) << 7) : static_cast<uint16_t>(0);
    #pragma unroll
                for (int i = 0; i < RPT; ++i) xg[(pt * RPT + i) * D + kc] = gcr[i] - m;
                if (pt == 3) vec[L::vGl + kc] = gcr[RPT - 1];
                if (trow >= 0 && trow / RPT == pt) vec[L::vGtr + kc] = gtr;
            }
            cbar();

            // ---- P2: factor tables; X = kn e^x, Y = qn e^x, Z = kn e^-x as bf16 hi/lo tiles ----
            for (int e = tid; e < 16 * D; e += kThreads) {
                const int r = e / D, k = e % D;
                if (r < 6) {
                    int I = (r < 1) ? 1 : (r < 3) ? 2 : 3;
                    const int J = r - I * (I - 1) / 2;
                    const float d = rintf((vec[L::vM + I * D + k] - vec[L::vM + J * D + k]) * kLog2e);   // <= 0
                    reinterpret_cast<uint16_t *>(vec + L::vFb)[r * D + k] =
                        d >= -126.f ? static_cast<uint16_t>((static_cast<int>(d) + 127) << 7) : static_cast<uint16_t>(0);
                } else if (r < 10) {
                    const int J = r - 6;
                    vec[L::vEglm + J * D + k] = ex2((vec[L::vGl + k] - vec[L::vM + J * D + k]) * kLog2e);
                } else if (r == 10) {
                    vec[L::vEgl + k] = ex2(vec[L::vGl + k] * kLog2e);
                } else if (track_here) {
                    if (r == 11) {
                        vec[L::vEtr + k] = ex2(vec[L::vGtr + k] * kLog2e);
                    } else {
                        const int J = r - 12;
                        vec[L::vEtrm + J * D + k] = ex2((vec[L::vGtr + k] - vec[L::vM + J * D + k]) * kLog2e);
                    }
                }
            }
            // The previous chunk's last products (o = QG S + Aqk v', the state
            // update) still read QG, KD and Aqk in the Y, Z and Aqk tiles this
            // chunk rewrites: wait for them (bars[3] tracks all three) before the
            // tiles below; the factor tables above touch none of them.
            if (!PREP && c > 0) {
                if (!mbar_wait(&bars[3], static_cast<uint32_t>((c - 1) & 1), p.status, abort_w) && tid == 0)
                    report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
                tc_fence_after();
            }
            for (int j = tid; j < BT * D / 8; j += kThreads) {
                const int row = j / (D / 8), c = 8 * (j % (D / 8));
                const float4 x0 = *reinterpret_cast<const float4 *>(xg + row * D + c);
                const float4 x1 = *reinterpret_cast<const float4 *>(xg + row * D + c + 4);
                const uint4 qq = *reinterpret_cast<const uint4 *>(rawQ + row * D + c);
                const uint4 kk = *reinterpret_cast<const uint4 *>(rawK + row * D + c);
                const float rq = vec[L::vRq + row], rk = vec[L::vRk + row];
                const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                const uint32_t qw[4] = {qq.x, qq.y, qq.z, qq.w}, kw[4] = {kk.x, kk.y, kk.z, kk.w};
                uint32_t xh[4], xl[4], yh[4], yl[4], zh[4], zl[4];
    #pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float t0 = xv[2 * e] * kLog2e, t1 = xv[2 * e + 1] * kLog2e;
                    const float E0 = ex2(t0), E1 = ex2(t1), F0 = ex2(-t0), F1 = ex2(-t1);
                    const float k0 = bf16_lo(kw[e]) * rk, k1 = bf16_hi(kw[e]) * rk;
                    const float q0 = bf16_lo(qw[e]) * rq, q1 = bf16_hi(qw[e]) * rq;
                    split2(k0 * E0, k1 * E1, xh[e], xl[e]);
                    split2(q0 * E0, q1 * E1, yh[e], yl[e]);
                    split2(k0 * F0, k1 * F1, zh[e], zl[e]);
                }
                const int o = f64(row, c);
                *reinterpret_cast<uint4 *>(Xh + o) = make_uint4(xh[0], xh[1], xh[2], xh[3]);
                *reinterpret_cast<uint4 *>(Xl + o) = make_uint4(xl[0], xl[1], xl[2], xl[3]);
                *reinterpret_cast<uint4 *>(Yh + o) = make_uint4(yh[0], yh[1], yh[2], yh[3]);
                *reinterpret_cast<uint4 *>(Yl + o) = make_uint4(yl[0], yl[1], yl[2], yl[3]);
                *reinterpret_cast<uint4 *>(Zh + o) = make_uint4(zh[0], zh[1], zh[2], zh[3]);
                *reinterpret_cast<uint4 *>(Zl + o) = make_uint4(zl[0], zl[1], zl[2], zl[3]);
            }
            cbar();

            // ---- P3: A' and Aqk, one 16x16 block pair per warp (T_II on diagonal ones) ----
            // Block (I, J) = X_I diag(e^{m_I - m_J}) Z_J^T: the factor is a power
            // of two, applied exactly to Z's bf16 hi/lo fragments.
            if (warp < 10) {
                int I, J;
                pair_ij(warp, I, J);
                const uint32_t *Fp =
                    (J < I) ? reinterpret_cast<const uint32_t *>(vec + L::vFb) + fslot(I, J) * (D / 2) : nullptr;
                float akk[2][4] = {}, aqk[2][4] = {};
    #pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    const int k0 = 16 * ks;
                    uint32_t xh[4], xl[4], yh[4], yl[4], zh[4], zl[4];
                    const uint32_t oa = 2 * fa_a(lane, 16 * I, k0), ob = 2 * fb_nk(lane, 16 * J, k0);
                    ldsm_x4(xh, s_base + L::kX + oa);
                    ldsm_x4(xl, s_base + L::kX + BT * D * 2 + oa);
                    ldsm_x4(yh, s_base + L::kY + oa);
                    ldsm_x4(yl, s_base + L::kY + BT * D * 2 + oa);
                    ldsm_x4(zh, s_base + L::kZ + ob);
                    ldsm_x4(zl, s_base + L::kZ + BT * D * 2 + ob);
                    if (Fp != nullptr) {
                        const uint32_t f0 = Fp[(k0 >> 1) + t4], f1 = Fp[(k0 >> 1) + 4 + t4];
                        zh[0] = bmul2(zh[0], f0);
                        zh[1] = bmul2(zh[1], f1);
                        zh[2] = bmul2(zh[2], f0);
                        zh[3] = bmul2(zh[3], f1);
                        zl[0] = bmul2(zl[0], f0);
                        zl[1] = bmul2(zl[1], f1);
                        zl[2] = bmul2(zl[2], f0);
                        zl[3] = bmul2(zl[3], f1);
                    }
                    mma3(akk[0], xh, xl, zh[0], zh[1], zl[0], zl[1]);
                    mma3(akk[1], xh, xl, zh[2], zh[3], zl[2], zl[3]);
                    mma3(aqk[0], yh, yl, zh[0], zh[1], zl[0], zl[1]);
                    mma3(aqk[1], yh, yl, zh[2], zh[3], zl[2], zl[3]);
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
                if (I == J) {
                    // T_II = (I + A'_II)^-1 at once: lane j (and j + 16, which
                    // repeats it) solves column j by forward substitution in fp32
                    // (entries above the diagonal are 0, so the unpredicated sums
                    // are exact).
                    __syncwarp();   // the block's A' rows are in shared memory
                    const int j = lane & 15;
                    float col[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float *arow = Ap + (16 * I + i) * AS + 16 * I;
                        float s0a = 0.f, s1a = 0.f;
#pragma unroll
                        for (int m = 0; m + 1 < i; m += 2) {
                            s0a = fmaf(arow[m], col[m], s0a);
                            s1a = fmaf(arow[m + 1], col[m + 1], s1a);
                        }
                        if (i & 1) s0a = fmaf(arow[i - 1], col[i - 1], s0a);
                        col[i] = (i == j) ? 1.f : (i > j ? -(s0a + s1a) : 0.f);
                    }
                    if (lane < 16) {
                        // T_II (fp32, for the off-diagonal blocks) and TB_II = T_II diag(beta)
                        // as bf16 hi/lo, the operand of u = TB v and W.
                        const float bj = vec[L::vBeta + 16 * I + j];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            Tm[(16 * I + i) * AS + 16 * I + j] = col[i];
                            uint16_t hi, lo;
                            split1(col[i] * bj, hi, lo);
                            TBh[swz<BT>(16 * I + i, 16 * I + j)] = hi;
                            TBl[swz<BT>(16 * I + i, 16 * I + j)] = lo;
                        }
                    }
                }
            } else if (o_pending) {
                // Warps 10..15, beside the block products: the previous chunk's
                // o tile leaves through the raw region's staging area (quadrants 0
                // and 1 have one warp each, 2 and 3 two).
                if (!mbar_wait(&bars[3], static_cast<uint32_t>((c - 1) & 1), p.status, abort_w) && lane == 0)
                    report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
                tc_fence_after();
                const bool pair = q4 >= 2;
                const int half = (warp >= 14) ? 1 : 0;
                o_cols(OstR, o_t0, o_n, pair ? 32 * half : 0, pair ? 32 : BT);
                fence_async_smem();
                nbar(3, 192);
                if (tid == 384) {
                    o_store(OstR, o_t0, o_n);
                    bulk_wait_read();   // before the next chunk's tiles land on the raw region
                }
            }
            cbar();

            // ---- P4: T = (I + A')^-1 on warps 0-3, beside the S split on warps 8-15 ----
            if (warp < 4) {
                // The diagonal blocks T_II came with P3. Off-diagonal blocks, 2x2
                // block-recursively: the inverse of [[M_A, 0], [A'_BA, M_B]] is
                // [[T_A, 0], [-T_B A'_BA T_A, T_B]].
                // Stage 1: T_10 and T_32 (the 32x32 diagonal halves); stage 2: the
                // lower-left 32x32 quadrant, one 16x16 block per warp. Every
                // product is split-bf16 (fp32 operands split into hi + lo).
                // B fragments of a fp32 16x16 block at (r0, c0) of a row-major
                // tile with row stride `ld`, columns [c0 + 8 nt, +8).
                auto bfrag = [&](const float *base, int ld, int r0, int c0, int nt, uint32_t &bh0, uint32_t &bh1,
                                 uint32_t &bl0, uint32_t &bl1) {
                    const float *b = base + (r0 + 2 * t4) * ld + c0 + 8 * nt + g;
                    split2(b[0], b[ld], bh0, bl0);
                    split2(b[8 * ld], b[9 * ld], bh1, bl1);
                };
                auto afrag = [&](const float *base, int ld, int r0, int c0, uint32_t (&ah)[4], uint32_t (&al)[4]) {
                    const float *a = base + (r0 + g) * ld + c0 + 2 * t4;
                    const float2 a0 = *reinterpret_cast<const float2 *>(a);
                    const float2 a1 = *reinterpret_cast<const float2 *>(a + 8 * ld);
                    const float2 a2 = *reinterpret_cast<const float2 *>(a + 8);
                    const float2 a3 = *reinterpret_cast<const float2 *>(a + 8 * ld + 8);
                    split2(a0.x, a0.y, ah[0], al[0]);
                    split2(a1.x, a1.y, ah[1], al[1]);
                    split2(a2.x, a2.y, ah[2], al[2]);
                    split2(a3.x, a3.y, ah[3], al[3]);
                };
                // acc[nt] += (16x16 block of `a` at (ar, ac)) x (block of `b` at (br, bc))
                auto blk = [&](float (&acc)[2][4], const float *a, int lda, int ar, int ac, const float *b, int ldb,
                               int br, int bc) {
                    uint32_t ah[4], al[4];
                    afrag(a, lda, ar, ac, ah, al);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        uint32_t bh0, bh1, bl0, bl1;
                        bfrag(b, ldb, br, bc, nt, bh0, bh1, bl0, bl1);
                        mma3(acc[nt], ah, al, bh0, bh1, bl0, bl1);
                    }
                };
                auto put = [&](float *dst, int ld, const float (&acc)[2][4], float sgn) {
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt) {
                        float *t = dst + g * ld + 8 * nt + 2 * t4;
                        *reinterpret_cast<float2 *>(t) = make_float2(sgn * acc[nt][0], sgn * acc[nt][1]);
                        *reinterpret_cast<float2 *>(t + 8 * ld) = make_float2(sgn * acc[nt][2], sgn * acc[nt][3]);
                    }
                };
                // -acc as block (r0, c0) of T, and of TB = T diag(beta) as bf16 hi/lo.
                auto put_t = [&](int r0, int c0, const float (&acc)[2][4]) {
                    put(Tm + r0 * AS + c0, AS, acc, -1.f);
#pragma unroll
                    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                        for (int hf = 0; hf < 2; ++hf) {
                            const int i = r0 + g + 8 * hf, j0 = c0 + 8 * nt + 2 * t4;
                            uint32_t hi, lo;
                            split2(-acc[nt][2 * hf] * vec[L::vBeta + j0], -acc[nt][2 * hf + 1] * vec[L::vBeta + j0 + 1],
                                   hi, lo);
                            *reinterpret_cast<uint32_t *>(TBh + swz<BT>(i, j0)) = hi;
                            *reinterpret_cast<uint32_t *>(TBl + swz<BT>(i, j0)) = lo;
                        }
                };
                float *const Pw = Pp + warp * 16 * L::PS;
                if (warp < 2) {
                    // T_IJ = -T_II (A'_IJ T_JJ), (I, J) = (1, 0) or (3, 2)
                    const int J = 2 * warp, I = J + 1;
                    float pacc[2][4] = {};
                    blk(pacc, Ap, AS, 16 * I, 16 * J, Tm, AS, 16 * J, 16 * J);
                    put(Pw, L::PS, pacc, 1.f);
                    __syncwarp();
                    float tacc[2][4] = {};
                    blk(tacc, Tm, AS, 16 * I, 16 * I, Pw, L::PS, 0, 0);
                    put_t(16 * I, 16 * J, tacc);
                }
                nbar(2, 128);
                {
                    // Block (r, cc) of the lower-left quadrant, r in {2, 3}, cc in {0, 1}:
                    // P_r,cc = sum_{m=cc}^{1} A'_r,m T_m,cc, then
                    // T_r,cc = -sum_{m=2}^{r} T_r,m P_m,cc (P_m,cc from warp 2 (m - 2) + cc).
                    const int r = 2 + (warp >> 1), cc = warp & 1;
                    float pacc[2][4] = {};
                    blk(pacc, Ap, AS, 16 * r, 16, Tm, AS, 16, 16 * cc);
                    if (cc == 0) blk(pacc, Ap, AS, 16 * r, 0, Tm, AS, 0, 0);
                    put(Pw, L::PS, pacc, 1.f);
                    nbar(2, 128);
                    float tacc[2][4] = {};
                    blk(tacc, Tm, AS, 16 * r, 32, Pp + cc * 16 * L::PS, L::PS, 0, 0);
                    if (r == 3) blk(tacc, Tm, AS, 48, 48, Pp + (2 + cc) * 16 * L::PS, L::PS, 0, 0);
                    put_t(16 * r, 16 * cc, tacc);
                }
            } else if (!PREP && warp >= 8) {
                // S^T -> bf16 hi/lo A operand and S^T <- S^T e^{gl} (deferred on a
                // tracked chunk): two warps per lane quadrant, half the columns each.
                if (c > 0) {
                    if (!mbar_wait(&bars[1], static_cast<uint32_t>((c - 1) & 1), p.status, abort_w) && lane == 0)
                        report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
                    tc_fence_after();
                }
                const int cb = ((warp >> 2) & 1) * (D / 2);
#pragma unroll
                for (int c16 = 0; c16 < D / 32; ++c16) {
                    const int col = cb + 16 * c16;
                    uint32_t r[16], hi[8], lo[8];
                    tmem_ld16(tq + kColS + col, r);
                    tmem_ld_wait();
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        split2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]), hi[e], lo[e]);
                    tmem_st8(tq + kColSH + col / 2, hi);
                    tmem_st8(tq + kColSL + col / 2, lo);
                    if (!track_here) {
                        const float4 *eg = reinterpret_cast<const float4 *>(vec + L::vEgl + col);
#pragma unroll
                        for (int e4 = 0; e4 < 4; ++e4) {
                            const float4 f = eg[e4];
                            r[4 * e4] = __float_as_uint(__uint_as_float(r[4 * e4]) * f.x);
                            r[4 * e4 + 1] = __float_as_uint(__uint_as_float(r[4 * e4 + 1]) * f.y);
                            r[4 * e4 + 2] = __float_as_uint(__uint_as_float(r[4 * e4 + 2]) * f.z);
                            r[4 * e4 + 3] = __float_as_uint(__uint_as_float(r[4 * e4 + 3]) * f.w);
                        }
                        tmem_st16(tq + kColS + col, r);
                    }
                }
                tmem_st_wait();
                tc_fence_before();
            }
            // TB came with the T blocks (P3's diagonal solves, P4's stages).
            fence_async_smem();   // TB tiles written by threads -> read by the tensor core
            cbar();
            if (!PREP && tid == 0) {
                mbar_arrive(sig_a);    // A' is dead: the next q tile may land
                mbar_arrive(&sig[0]);  // u = TB v may start
            }
            if (has_next) load_beta(c + 1);

            // ---- P7 (warps 0..D/16-1): W = TB (kn e^{gc}), 16 key columns per warp ----
            // kn e^{gc} = X e^{m_I}: X's bf16 hi/lo fragments scaled exactly by
            // 2^{m_I / ln 2}. The other warps run P8 meanwhile (disjoint tiles).
            constexpr int NW7 = D / 16;
            if (warp < NW7) {
                float wacc[4][2][4] = {};
                const uint16_t *sv16 = reinterpret_cast<const uint16_t *>(vec + L::vS);
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    uint32_t kbh[4], kbl[4];
                    const uint32_t ob = 2 * f64(16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3), 16 * warp + ((lane >> 4) << 3));
                    ldsm_x4_t(kbh, s_base + L::kX + ob);
                    ldsm_x4_t(kbl, s_base + L::kX + BT * D * 2 + ob);
                    const uint32_t s0 = static_cast<uint32_t>(sv16[ks * D + 16 * warp + g]) * 0x10001u;
                    const uint32_t s1 = static_cast<uint32_t>(sv16[ks * D + 16 * warp + 8 + g]) * 0x10001u;
                    kbh[0] = bmul2(kbh[0], s0);
                    kbh[1] = bmul2(kbh[1], s0);
                    kbh[2] = bmul2(kbh[2], s1);
                    kbh[3] = bmul2(kbh[3], s1);
                    kbl[0] = bmul2(kbl[0], s0);
                    kbl[1] = bmul2(kbl[1], s0);
                    kbl[2] = bmul2(kbl[2], s1);
                    kbl[3] = bmul2(kbl[3], s1);
#pragma unroll
                    for (int mt = ks; mt < 4; ++mt) {
                        uint32_t ah[4], al[4];
                        ldsm_x4(ah, s_base + L::kTBh + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
                        ldsm_x4(al, s_base + L::kTBl + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
                        mma3(wacc[mt][0], ah, al, kbh[0], kbh[1], kbl[0], kbl[1]);
                        mma3(wacc[mt][1], ah, al, kbh[2], kbh[3], kbl[2], kbl[3]);
                    }
                }
                nbar(4, 32 * NW7);   // X fully consumed: W replaces it
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
                            *reinterpret_cast<uint32_t *>(Wh + f64(j, kcol)) = hi;
                            *reinterpret_cast<uint32_t *>(Wl + f64(j, kcol)) = lo;
                        }
                if constexpr (PREP) {
                    // u = TB v for value columns [16w, 16w + 16) (v is exact in bf16:
                    // two products), stored negated in the record's layout in the
                    // gate region (consumed in P2).
                    float uacc[4][2][4] = {};
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        uint32_t vb[4];
                        ldsm_x4_t(vb, s_base + L::kV +
                                          2 * f64(16 * ks + (lane & 7) + (((lane >> 3) & 1) << 3),
                                                  16 * warp + ((lane >> 4) << 3)));
#pragma unroll
                        for (int mt = ks; mt < 4; ++mt) {
                            uint32_t ah[4], al[4];
                            ldsm_x4(ah, s_base + L::kTBh + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
                            ldsm_x4(al, s_base + L::kTBl + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
                            mma16816(uacc[mt][0], al, vb[0], vb[1]);
                            mma16816(uacc[mt][0], ah, vb[0], vb[1]);
                            mma16816(uacc[mt][1], al, vb[2], vb[3]);
                            mma16816(uacc[mt][1], ah, vb[2], vb[3]);
                        }
                    }
                    float *ust = reinterpret_cast<float *>(sm + L::kRawG);
#pragma unroll
                    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
                        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                            for (int hf = 0; hf < 2; ++hf) {
                                const int t = 16 * mt + g + 8 * hf, v0 = 16 * warp + 8 * nt + 2 * t4;
                                ust[((t >> 2) * D + v0) * 4 + (t & 3)] = -uacc[mt][nt][2 * hf];
                                ust[((t >> 2) * D + v0 + 1) * 4 + (t & 3)] = -uacc[mt][nt][2 * hf + 1];
                            }
                }
            // ---- P8: QG = Y e^{m_I} (exact), KD = Z e^{gl - m_J}, tracked K_r; in place ----
            } else {
                for (int j = tid - 32 * NW7; j < BT * D / 8; j += kThreads - 32 * NW7) {
                    const int row = j / (D / 8), c = 8 * (j % (D / 8)), blk = row >> 4;
                    const int o = f64(row, c);
                    {
                        const uint4 sc = *reinterpret_cast<const uint4 *>(
                            reinterpret_cast<const uint16_t *>(vec + L::vS) + blk * D + c);
                        const uint4 hq = *reinterpret_cast<const uint4 *>(QGh + o);
                        const uint4 lq = *reinterpret_cast<const uint4 *>(QGl + o);
                        *reinterpret_cast<uint4 *>(QGh + o) =
                            make_uint4(bmul2(hq.x, sc.x), bmul2(hq.y, sc.y), bmul2(hq.z, sc.z), bmul2(hq.w, sc.w));
                        *reinterpret_cast<uint4 *>(QGl + o) =
                            make_uint4(bmul2(lq.x, sc.x), bmul2(lq.y, sc.y), bmul2(lq.z, sc.z), bmul2(lq.w, sc.w));
                    }
                    uint4 h = *reinterpret_cast<const uint4 *>(KDh + o);
                    uint4 l = *reinterpret_cast<const uint4 *>(KDl + o);
                    const uint32_t hw[4] = {h.x, h.y, h.z, h.w}, lw[4] = {l.x, l.y, l.z, l.w};
                    const float4 eg0 = *reinterpret_cast<const float4 *>(vec + L::vEglm + blk * D + c);
                    const float4 eg1 = *reinterpret_cast<const float4 *>(vec + L::vEglm + blk * D + c + 4);
                    const float eg[8] = {eg0.x, eg0.y, eg0.z, eg0.w, eg1.x, eg1.y, eg1.z, eg1.w};
                    float z[8];
    #pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        z[2 * e] = bf16_lo(hw[e]) + bf16_lo(lw[e]);
                        z[2 * e + 1] = bf16_hi(hw[e]) + bf16_hi(lw[e]);
                    }
                    uint32_t dh[4], dl[4];
    #pragma unroll
                    for (int e = 0; e < 4; ++e) split2(z[2 * e] * eg[2 * e], z[2 * e + 1] * eg[2 * e + 1], dh[e], dl[e]);
                    *reinterpret_cast<uint4 *>(KDh + o) = make_uint4(dh[0], dh[1], dh[2], dh[3]);
                    *reinterpret_cast<uint4 *>(KDl + o) = make_uint4(dl[0], dl[1], dl[2], dl[3]);
                    if (track_here) {
                        const float4 et0 = *reinterpret_cast<const float4 *>(vec + L::vEtrm + blk * D + c);
                        const float4 et1 = *reinterpret_cast<const float4 *>(vec + L::vEtrm + blk * D + c + 4);
                        const float et[8] = {et0.x, et0.y, et0.z, et0.w, et1.x, et1.y, et1.z, et1.w};
                        const bool live = row < rtrack;
    #pragma unroll
                        for (int e = 0; e < 4; ++e)
                            split2(live ? z[2 * e] * et[2 * e] : 0.f, live ? z[2 * e + 1] * et[2 * e + 1] : 0.f, dh[e],
                                   dl[e]);
                        *reinterpret_cast<uint4 *>(KRh + o) = make_uint4(dh[0], dh[1], dh[2], dh[3]);
                        *reinterpret_cast<uint4 *>(KRl + o) = make_uint4(dl[0], dl[1], dl[2], dl[3]);
                    }
                }
            }
            fence_async_smem();   // tiles written by threads -> read by the tensor core
            cbar();
            if constexpr (PREP) {
                // The chunk-head's scan operands -> its record (and the tracked
                // prefix operand -> the request's), one bulk copy per part.
                if (tid == 0) {
                    using R = Rec<D>;
                    const int hl = h - p.head_begin;
                    uint8_t *rc = rec + (static_cast<int64_t>(cbase[req] + c) * p.head_count + hl) * R::kBytes;
                    bulk_s2g(rc + R::kW, sm + L::kX, BT * D * 4);
                    bulk_s2g(rc + R::kQG, sm + L::kY, BT * D * 4);
                    bulk_s2g(rc + R::kKD, sm + L::kZ, BT * D * 4);
                    bulk_s2g(rc + R::kU, sm + L::kRawG, BT * D * 4);
                    bulk_s2g(rc + R::kAQ, sm + L::kAQh, BT * BT * 4);
                    bulk_s2g(rc + R::kEgl, vec + L::vEgl, D * 4);
                    if (track_here) {
                        uint8_t *tr = trec + (static_cast<int64_t>(req) * p.head_count + hl) * R::tBytes;
                        bulk_s2g(tr + R::tKR, sm + L::kRawQ, BT * D * 4);
                        bulk_s2g(tr + R::tEtr, vec + L::vEtr, D * 4);
                    }
                    bulk_commit();
                    bulk_wait_read();   // smem may be released; the kernel's end publishes the writes
                }
                continue;
            }
            if (tid == 0) mbar_arrive(&sig[1]);   // W, QG, KD (and K_r) are in place: W S and QG S may start

            // ---- P9: the state scan: -v'^T (fp32) -> v'^T hi/lo A operand, 16 columns per warp ----
            if (!mbar_wait(&bars[0], static_cast<uint32_t>(c & 1), p.status, abort_w) && tid == 0)
                report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            tc_fence_after();
            {
                uint32_t r[16], hi[8], lo[8];
                tmem_ld16(tq + kColNU + 16 * cs, r);
                tmem_ld_wait();
    #pragma unroll
                for (int e = 0; e < 8; ++e)
                    split2(-__uint_as_float(r[2 * e]), -__uint_as_float(r[2 * e + 1]), hi[e], lo[e]);
                tmem_st8(tq + kColVH + 8 * cs, hi);
                tmem_st8(tq + kColVL + 8 * cs, lo);
            }
            // Tracked prefix: S^T e^{gc_{r-1}} into the S hi/lo columns (consumed:
            // their last reader finished before bars[0]), then the deferred S^T e^{gl}.
            if (track_here) {
                uint32_t r[SC], t[SC];
                tmem_ld<SC>(tq + kColS + SC * cs, r);
                tmem_ld_wait();
    #pragma unroll
                for (int e = 0; e < SC; ++e) {
                    t[e] = __float_as_uint(__uint_as_float(r[e]) * vec[L::vEtr + SC * cs + e]);
                    r[e] = __float_as_uint(__uint_as_float(r[e]) * vec[L::vEgl + SC * cs + e]);
                }
                tmem_st<SC>(tq + kColTR + SC * cs, t);
                tmem_st<SC>(tq + kColS + SC * cs, r);
            }
            tmem_st_wait();
            tc_fence_before();
            cbar();
            if (tid == 0) mbar_arrive(&sig[2]);   // the state update and o += Aqk v' may start
            if (track_here) {
                // A tracked chunk finishes here: the checkpoint leaves tensor memory
                // before the next S split reuses its columns; the o tile goes too.
                if (!mbar_wait(&bars[3], static_cast<uint32_t>(c & 1), p.status, abort_w) && tid == 0)
                    report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
                tc_fence_after();
                o_cols(OstX, t0, n, 16 * cs, 16);
                fence_async_smem();
                cbar();
                if (tid == 0) {
                    o_store(OstX, t0, n);
                    ox_busy = true;
                }
                float *ts = p.state + tslot * s0 + h * s1;
                uint32_t r[SC];
                tmem_ld<SC>(tq + kColTR + SC * cs, r);
                tmem_ld_wait();
                if (srow < D) {
    #pragma unroll
                    for (int e = 0; e < SC; ++e) ts[srow * sv + (SC * cs + e) * sk] = __uint_as_float(r[e]);
                }
                o_pending = false;
            } else {
                o_pending = true;
                o_t0 = t0;
                o_n = n;
            }
            }   // chunk loop

        if (!PREP && nchunks > 0) {
            const uint32_t lph = static_cast<uint32_t>((nchunks - 1) & 1);
            if (o_pending) {
                if (!mbar_wait(&bars[3], lph, p.status, abort_w) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
                tc_fence_after();
                o_cols(OstX, o_t0, o_n, 16 * cs, 16);
                fence_async_smem();
                cbar();
                if (tid == 0) o_store(OstX, o_t0, o_n);
            }
            if (!mbar_wait(&bars[1], lph, p.status, abort_w) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            tc_fence_after();
        }
        // Final state S^T -> pool slot (padding slot 0 is never written).
        if (!PREP) {
            float *hs = p.state + slot * s0 + h * s1;
            uint32_t r[SC];
            tmem_ld<SC>(tq + kColS + SC * cs, r);
            tmem_ld_wait();
            if (slot > 0 && srow < D) {
#pragma unroll
                for (int e = 0; e < SC; ++e) hs[srow * sv + (SC * cs + e) * sk] = __uint_as_float(r[e]);
            }
        }
        if (tid == 0 || tid == 384) bulk_wait_read();   // output stores have read their staging tiles
    }
    // After an expired wait the CTA's waits gave up early: before the CTA
    // frees its tensor memory and exits, thread 0 waits (bounded, without the
    // shortcut) for the last chunk's tile copies and tensor-core products,
    // which complete every earlier phase of their barriers.
    if (*abort_w != 0 && tid == 0 && nchunks > 0) {
        const uint32_t lph = PREP ? 0u : static_cast<uint32_t>((nchunks - 1) & 1);
        mbar_wait(&bars[2], lph, nullptr);
        if (!PREP) {
            mbar_wait(&bars[1], lph, nullptr);
            mbar_wait(&bars[3], lph, nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (!PREP && warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Split path, part 2: the inter-chunk scan alone. One CTA per (sequence,
// head). The producer thread streams each chunk's record (written by the
// prep kernel) into the operand slots of shared memory as soon as the
// previous chunk's product reading a slot has completed, and issues the two
// state products (W S onto -u, the state update); the compute warps split the
// state (and leave the split for the output kernel) and convert v'. Per chunk
// the serial chain is: S split -> W S -> v' conversion -> state update; the
// stores and the next chunk's -u^T copy run beside the products.
// ---------------------------------------------------------------------------
template <int D>
__global__ void __launch_bounds__(kThreads + 32, 1)
    chunk_scan_kernel(const KdaArgs p, const int32_t *plan, int phase, const __grid_constant__ TmaMaps maps,
                      const uint8_t *rec, const uint8_t *trec, const int32_t *cbase, uint8_t *sout, float *states) {
    using L = Smem<D>;
    using R = Rec<D>;
    constexpr int KS = D / 16;
    constexpr int SC = D / 4;                        // state columns per slice
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    // -u^T slots (record layout), chunk c in slot c & 1
    const float *const Us0 = reinterpret_cast<const float *>(sm + L::kRawG);
    const float *const Us1 = reinterpret_cast<const float *>(sm + L::kY);
    float *const vec = reinterpret_cast<float *>(sm + L::kVec);
    uint64_t *const mb = reinterpret_cast<uint64_t *>(sm + L::kBar);
    // product completions
    uint64_t *const bG2 = mb + 1, *const bG4 = mb + 3;
    // operand-slot loads
    uint64_t *const lU0 = mb + 5, *const lU1 = mb + 4, *const lEgl = mb + 6, *const lW = mb + 7, *const lKD = mb + 9, *const lTR = mb + 11;
    // compute warps -> producer
    uint64_t *const sSplit = mb + 12, *const sConv = mb + 13;
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(sm + L::kBar + 120);
    volatile int32_t *const abort_w = reinterpret_cast<volatile int32_t *>(sm + L::kBar + 124);   // give-up word
    const uint32_t s_base = smem_addr(sm);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ti = blockIdx.x / p.head_count;
    const int hl = blockIdx.x % p.head_count, h = p.head_begin + hl;
    if (ti >= plan[1 + phase]) return;
    const PlanView pv(const_cast<int32_t *>(plan), p.num_req, plan[3]);
    const int32_t task = pv.tasks(phase)[ti];
    const int req = task & 1023, kind = (task >> 10) & 3, half = (task >> 12) & 1, seg = task >> 13;
    const int nseg = pv.segs()[req], seglen = pv.seglen()[req];
    const bool truth = kind == kTaskTrue;
    const int slot_cap = plan[0];
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
    if (p.track_indices != nullptr && truth) {
        tslot = load_index(p.track_indices, p.index_bytes[2], req);
        if (tslot < 0 || tslot >= p.num_slots) {
            if (tid == 0) report(p.status, KDA_DEVICE_ERR_BAD_SLOT);
            return;
        }
        if (tslot > 0) tlen = load_index(p.track_lens, p.index_bytes[3], req);
    }
    // This task's chunks [c0, c0 + nchunks) of the request (below, chunk
    // indices are relative to c0). Segment `seg` spans [seg L, seg L + len);
    // its midpoint is `mid` chunks in. A first-pass chain covers the segment
    // (or, with `half`, its first half) and leaves its state at the midpoint;
    // a rescan half covers [0, mid) or [mid, len) of the segment.
    const int req_chunks = static_cast<int>((eos - bos + BT - 1) / BT);
    const int seg0 = seg * seglen;
    const int seg_len = max(0, min(req_chunks, seg0 + seglen) - seg0);
    const int mid = (seg_len + 1) / 2;
    const bool rescan2 = truth && seg > 0 && half;          // second half of a rescan
    const int c0 = rescan2 ? seg0 + mid : seg0;
    const int nchunks = truth ? (seg == 0 ? seg_len : (half ? seg_len - mid : mid)) : (half ? mid : seg_len);
    const int mid_at = truth ? -1 : mid;                    // local chunk of the midpoint state
    const int64_t s0 = p.state_stride[0], s1 = p.state_stride[1], sk = p.state_stride[2], sv = p.state_stride[3];
    auto trk_at = [&](int c) {
        const int64_t rt = tlen - static_cast<int64_t>(c0 + c) * BT;
        return tslot > 0 && rt > 0 && rt <= BT;
    };
    auto rec_of = [&](int c) {
        return rec + (static_cast<int64_t>(cbase[req] + c0 + c) * p.head_count + hl) * R::kBytes;
    };
    auto sout_of = [&](int c) {
        return sout + (static_cast<int64_t>(cbase[req] + c0 + c) * p.head_count + hl) * ScanOut<D>::kBytes;
    };
    // Exchange slots of this request's segment boundaries (segment sg >= 1).
    auto xslot = [&](int which, int sg) {
        return state_slot<D>(states, slot_cap, p.head_count, which, pv.sbase()[req] + sg - 1, hl);
    };
    const bool use_u = kind != kTaskIdent;
    const uint8_t *trk_rec = trec + (static_cast<int64_t>(req) * p.head_count + hl) * R::tBytes;

    if (warp == 0) tmem_alloc(tmem_slot, kTmemCols);
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 15; ++i) mbar_init(&mb[i], 1);
        *abort_w = 0;
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int q4 = warp & 3, cs = warp >> 2;
    const int srow = 32 * q4 + lane;
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q4) << 16);

    if (warp == kThreads / 32) {
        // ===== producer =====
        constexpr uint32_t id_kd = idesc_bf16(128, D, false, true, false);
        if (lane == 0 && rescan2) {
            // S_mid^T = S_start^T A_mid^T + B_mid^T: the compute warps staged
            // S_start^T's split (tensor memory), B_mid^T (the accumulator) and
            // A_mid^T as MN-major hi/lo tiles in the W and KD slots.
            if (!mbar_wait(mb + 14, 0, p.status, abort_w)) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < KS; ++kk) {
                const uint32_t ah = tmem + kColSH + 8 * kk, al = tmem + kColSL + 8 * kk;
                const uint64_t xh = sdesc(s_base + L::kX + kk * 2048, D * 128, 1024);
                const uint64_t xl = sdesc(s_base + L::kZ + kk * 2048, D * 128, 1024);
                umma_ts(tmem + kColS, al, xh, id_kd, 1u);
                umma_ts(tmem + kColS, ah, xl, id_kd, 1u);
                umma_ts(tmem + kColS, ah, xh, id_kd, 1u);
            }
            umma_commit(mb + 0);
            // the W and KD slots take their records once the product is done
            if (!mbar_wait(mb + 0, 0, p.status, abort_w)) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
        }
        if (lane == 0 && nchunks > 0) {
            constexpr uint32_t id_n64 = idesc_bf16(128, 64, false, false, false);
            auto pwait = [&](uint64_t *b, uint32_t ph) {
                if (!mbar_wait(b, ph, p.status, abort_w)) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            };
            auto load = [&](uint64_t *bar, void *dst, const uint8_t *src, uint32_t bytes) {
                mbar_arrive_expect_tx(bar, bytes);
                bulk_g2s(dst, src, bytes, bar);
            };
            auto load_tr = [&] {
                mbar_arrive_expect_tx(lTR, BT * D * 4 + D * 4);
                bulk_g2s(sm + L::kRawQ, trk_rec + R::tKR, BT * D * 4, lTR);
                bulk_g2s(vec + L::vEtr, trk_rec + R::tEtr, D * 4, lTR);
            };
            if (use_u) {
                load(lU0, sm + L::kRawG, rec_of(0) + R::kU, BT * D * 4);
                if (nchunks > 1) load(lU1, sm + L::kY, rec_of(1) + R::kU, BT * D * 4);
            }
            load(lEgl, vec + L::vEgl, rec_of(0) + R::kEgl, D * 4);
            load(lW, sm + L::kX, rec_of(0) + R::kW, BT * D * 4);
            load(lKD, sm + L::kZ, rec_of(0) + R::kKD, BT * D * 4);
            if (trk_at(0)) load_tr();
            uint32_t trph = 0;
            for (int c = 0; c < nchunks; ++c) {
                const uint32_t ph = static_cast<uint32_t>(c & 1);
                const bool trk = trk_at(c), nxt = c + 1 < nchunks;
                // NU (= -u^T, set by the compute warps with the split) += (W S)^T
                // -> -v'^T, once the state is split and W landed.
                pwait(sSplit, ph);
                // -u^T of chunk c was copied into NU before the split: its slot
                // takes chunk c + 2.
                if (use_u && c + 2 < nchunks)
                    load((c & 1) ? lU1 : lU0, sm + ((c & 1) ? L::kY : L::kRawG), rec_of(c + 2) + R::kU, BT * D * 4);
                pwait(lW, ph);
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < KS; ++kk) {
                    const uint32_t ah = tmem + kColSH + 8 * kk, al = tmem + kColSL + 8 * kk;
                    const uint32_t off = (kk >> 2) * 8192 + (kk & 3) * 32;
                    const uint64_t wh = sdesc(s_base + L::kX + off, 16, 1024);
                    const uint64_t wl = sdesc(s_base + L::kX + BT * D * 2 + off, 16, 1024);
                    umma_ts(tmem + kColNU, al, wh, id_n64, 1u);
                    umma_ts(tmem + kColNU, ah, wl, id_n64, 1u);
                    umma_ts(tmem + kColNU, ah, wh, id_n64, 1u);
                }
                umma_commit(bG2);
                // W of the next chunk as soon as W S has completed: it is the first
                // operand the next chunk's chain needs.
                if (nxt) {
                    pwait(bG2, ph);
                    load(lW, sm + L::kX, rec_of(c + 1) + R::kW, BT * D * 4);
                }
                // S^T += v'^T KD (and the tracked prefix).
                pwait(sConv, ph);
                // e^{gl} of the next chunk: this one's was last read before sConv.
                if (nxt) load(lEgl, vec + L::vEgl, rec_of(c + 1) + R::kEgl, D * 4);
                pwait(lKD, ph);
                if (trk) pwait(lTR, trph);
                tc_fence_after();
#pragma unroll
                for (int kk = 0; kk < 4; ++kk) {
                    const uint32_t ah = tmem + kColVH + 8 * kk, al = tmem + kColVL + 8 * kk;
                    const uint64_t dh = sdesc(s_base + L::kZ + kk * 2048, 8192, 1024);
                    const uint64_t dl = sdesc(s_base + L::kZ + BT * D * 2 + kk * 2048, 8192, 1024);
                    umma_ts(tmem + kColS, al, dh, id_kd, 1u);
                    umma_ts(tmem + kColS, ah, dl, id_kd, 1u);
                    umma_ts(tmem + kColS, ah, dh, id_kd, 1u);
                    if (trk) {
                        const uint64_t rh = sdesc(s_base + L::kRawQ + kk * 2048, 8192, 1024);
                        const uint64_t rl = sdesc(s_base + L::kRawK + kk * 2048, 8192, 1024);
                        umma_ts(tmem + kColTR, al, rh, id_kd, 1u);
                        umma_ts(tmem + kColTR, ah, rl, id_kd, 1u);
                        umma_ts(tmem + kColTR, ah, rh, id_kd, 1u);
                    }
                }
                umma_commit(bG4);
                if (trk) trph ^= 1u;
                if (nxt) {
                    pwait(bG4, ph);
                    load(lKD, sm + L::kZ, rec_of(c + 1) + R::kKD, BT * D * 4);
                    if (trk_at(c + 1)) load_tr();
                }
            }
        }
    } else {
        // ===== compute warps 0..15 =====
        auto cbar = [] { nbar(1, kThreads); };
        // Initial state S^T -> tensor memory: the pool slot (a length-0
        // checkpoint is the initial state), a segment's exchanged start state,
        // zero, or the identity.
        if (rescan2) {
            // Second half of a rescanned segment: stage the operands of
            // S_mid^T = S_start^T A_mid^T + B_mid^T for the producer.
            const bool row_ok = srow < D;
            uint32_t r[SC], hi[SC / 2], lo[SC / 2];
            auto load_row = [&](const float *src) {
#pragma unroll
                for (int e = 0; e < SC / 4; ++e) {
                    const float4 x = row_ok ? *reinterpret_cast<const float4 *>(src + ((SC / 4 * cs + e) * D + srow) * 4)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
                    r[4 * e] = __float_as_uint(x.x);
                    r[4 * e + 1] = __float_as_uint(x.y);
                    r[4 * e + 2] = __float_as_uint(x.z);
                    r[4 * e + 3] = __float_as_uint(x.w);
                }
            };
            load_row(xslot(kSlotStart, seg));
#pragma unroll
            for (int e = 0; e < SC / 2; ++e)
                split2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]), hi[e], lo[e]);
            tmem_st<SC / 2>(tq + kColSH + (SC / 2) * cs, hi);
            tmem_st<SC / 2>(tq + kColSL + (SC / 2) * cs, lo);
            load_row(xslot(kSlotBmid, seg));
            tmem_st<SC>(tq + kColS + SC * cs, r);
            // A_mid^T (rows j, columns k) -> swizzled bf16 hi/lo tiles, 64-column
            // blocks of D rows x 128 B: hi in the W slot, lo in the KD slot.
            const float *am = xslot(kSlotAmid, seg);
#pragma unroll
            for (int e = 0; e < D * D / 4 / kThreads; ++e) {
                const int q = tid + kThreads * e, j = q % D, k = 4 * (q / D);
                const float4 x = *reinterpret_cast<const float4 *>(am + static_cast<int64_t>(q) * 4);
                uint32_t h0, h1, l0, l1;
                split2(x.x, x.y, h0, l0);
                split2(x.z, x.w, h1, l1);
                const int o = ((k >> 6) * (D * 64) + swz<64>(j, k & 63)) * 2;
                *reinterpret_cast<uint2 *>(sm + L::kX + o) = make_uint2(h0, h1);
                *reinterpret_cast<uint2 *>(sm + L::kZ + o) = make_uint2(l0, l1);
            }
            fence_async_smem();
            tmem_st_wait();
            tc_fence_before();
            nbar(1, kThreads);
            if (tid == 0) mbar_arrive(mb + 14);
            if (!mbar_wait(mb + 0, 0, p.status, abort_w) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            tc_fence_after();
        } else {
            const bool row_ok = srow < D;
            uint32_t r[SC];
            if (truth && seg == 0) {
                const float *hs = p.state + slot * s0 + h * s1;
                float *ts = p.state + tslot * s0 + h * s1;
#pragma unroll
                for (int e = 0; e < SC; ++e) {
                    const int k = SC * cs + e;
                    const float x = (slot > 0 && row_ok) ? hs[srow * sv + k * sk] : 0.f;
                    r[e] = __float_as_uint(x);
                    if (row_ok && tslot > 0 && tlen == 0) ts[srow * sv + k * sk] = x;
                }
            } else if (truth) {
                const float *xs = xslot(0, seg);
#pragma unroll
                for (int e = 0; e < SC / 4; ++e) {
                    const float4 x = row_ok ? *reinterpret_cast<const float4 *>(xs + ((SC / 4 * cs + e) * D + srow) * 4)
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
                    r[4 * e] = __float_as_uint(x.x);
                    r[4 * e + 1] = __float_as_uint(x.y);
                    r[4 * e + 2] = __float_as_uint(x.z);
                    r[4 * e + 3] = __float_as_uint(x.w);
                }
            } else {
#pragma unroll
                for (int e = 0; e < SC; ++e)
                    r[e] = __float_as_uint(kind == kTaskIdent && row_ok && SC * cs + e == srow ? 1.f : 0.f);
            }
            tmem_st<SC>(tq + kColS + SC * cs, r);
            tmem_st_wait();
        }
        auto cwait = [&](uint64_t *bar, uint32_t phase) {
            if (!mbar_wait(bar, phase, p.status, abort_w) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
        };
        // NU <- -u^T of chunk c (this warp's 16 token columns of value row srow);
        // the copy reaches G2 through the wait, fence and barrier before sSplit.
        // A transfer chain (identity start) has u = 0.
        auto init_nu = [&](int c) {
            if (use_u) cwait((c & 1) ? lU1 : lU0, static_cast<uint32_t>((c >> 1) & 1));
            const float *us = (c & 1) ? Us1 : Us0;
            uint32_t r[16];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 u4 = use_u && srow < D
                                      ? *reinterpret_cast<const float4 *>(us + ((4 * cs + k) * D + srow) * 4)
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
                r[4 * k] = __float_as_uint(u4.x);
                r[4 * k + 1] = __float_as_uint(u4.y);
                r[4 * k + 2] = __float_as_uint(u4.z);
                r[4 * k + 3] = __float_as_uint(u4.w);
            }
            tmem_st16(tq + kColNU + 16 * cs, r);
        };
        if (nchunks > 0) init_nu(0);
        uint32_t trph = 0;
        for (int c = 0; c < nchunks; ++c) {
            const uint32_t ph = static_cast<uint32_t>(c & 1);
            const bool trk = trk_at(c);
            // (1) S^T -> bf16 hi/lo A operand of W S: the only work between the
            // state update of chunk c - 1 and the producer's next product.
            if (c > 0) cwait(bG4, static_cast<uint32_t>((c - 1) & 1));
            tc_fence_after();
            uint32_t r[SC], hi[SC / 2], lo[SC / 2];
            tmem_ld<SC>(tq + kColS + SC * cs, r);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < SC / 2; ++e)
                split2(__uint_as_float(r[2 * e]), __uint_as_float(r[2 * e + 1]), hi[e], lo[e]);
            tmem_st<SC / 2>(tq + kColSH + (SC / 2) * cs, hi);
            tmem_st<SC / 2>(tq + kColSL + (SC / 2) * cs, lo);
            tmem_st_wait();
            tc_fence_before();
            cbar();
            if (tid == 0) mbar_arrive(sSplit);   // S split, NU = -u^T, -u^T slot read
            // (2) while W S runs: the chunk-start state for the output kernel,
            // (value row, keys), and S^T <- S^T e^{gl} (deferred on a tracked chunk).
            if (truth && srow < D) {
                uint16_t *sh = reinterpret_cast<uint16_t *>(sout_of(c) + ScanOut<D>::kSH);
                uint16_t *sl = reinterpret_cast<uint16_t *>(sout_of(c) + ScanOut<D>::kSL);
#pragma unroll
                for (int q8 = 0; q8 < SC / 8; ++q8) {
                    const int o = fr<D>(srow, SC * cs + 8 * q8);
                    *reinterpret_cast<uint4 *>(sh + o) =
                        make_uint4(hi[4 * q8], hi[4 * q8 + 1], hi[4 * q8 + 2], hi[4 * q8 + 3]);
                    *reinterpret_cast<uint4 *>(sl + o) =
                        make_uint4(lo[4 * q8], lo[4 * q8 + 1], lo[4 * q8 + 2], lo[4 * q8 + 3]);
                }
            }
            // A first-pass chain leaves the state at its segment's midpoint.
            if (c == mid_at && srow < D) {
                float *xs = xslot(kind + 2, seg);
#pragma unroll
                for (int e = 0; e < SC / 4; ++e)
                    *reinterpret_cast<float4 *>(xs + ((SC / 4 * cs + e) * D + srow) * 4) =
                        make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                    __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
            }
            cwait(lEgl, ph);
            if (!trk) {
                const float *eg = vec + L::vEgl + SC * cs;
#pragma unroll
                for (int e = 0; e < SC; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * eg[e]);
                tmem_st<SC>(tq + kColS + SC * cs, r);
            }
            // (3) -v'^T (fp32) -> v'^T hi/lo A operand of the state update.
            cwait(bG2, ph);
            tc_fence_after();
            uint32_t v[16], vh[8], vl[8];
            tmem_ld16(tq + kColNU + 16 * cs, v);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 8; ++e)
                split2(-__uint_as_float(v[2 * e]), -__uint_as_float(v[2 * e + 1]), vh[e], vl[e]);
            tmem_st8(tq + kColVH + 8 * cs, vh);
            tmem_st8(tq + kColVL + 8 * cs, vl);
            if (trk) {
                // S^T e^{gc_{r-1}} into the S hi/lo columns (W S, their last
                // reader, has completed), then the deferred S^T e^{gl}.
                cwait(lTR, trph);
                uint32_t t[SC];
#pragma unroll
                for (int e = 0; e < SC; ++e) {
                    t[e] = __float_as_uint(__uint_as_float(r[e]) * vec[L::vEtr + SC * cs + e]);
                    r[e] = __float_as_uint(__uint_as_float(r[e]) * vec[L::vEgl + SC * cs + e]);
                }
                tmem_st<SC>(tq + kColTR + SC * cs, t);
                tmem_st<SC>(tq + kColS + SC * cs, r);
            }
            tmem_st_wait();
            tc_fence_before();
            cbar();
            if (tid == 0) mbar_arrive(sConv);   // v' split, S^T e^{gl} (and the checkpoint operand) stored
            // (4) while the state update runs: -u^T of the next chunk into NU
            // (the conversion above was its last reader).
            if (c + 1 < nchunks) init_nu(c + 1);
            if (trk) {
                // The checkpoint leaves tensor memory before the next split
                // reuses its columns (the barrier orders every warp's read
                // before any warp's next split).
                cwait(bG4, ph);
                tc_fence_after();
                float *ts = p.state + tslot * s0 + h * s1;
                uint32_t t[SC];
                tmem_ld<SC>(tq + kColTR + SC * cs, t);
                tmem_ld_wait();
                if (srow < D) {
#pragma unroll
                    for (int e = 0; e < SC; ++e) ts[srow * sv + (SC * cs + e) * sk] = __uint_as_float(t[e]);
                }
                trph ^= 1u;
                tc_fence_before();
                cbar();
            }
        }
        if (nchunks > 0) {
            if (!mbar_wait(bG4, static_cast<uint32_t>((nchunks - 1) & 1), p.status, abort_w) && tid == 0)
                report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
            tc_fence_after();
        }
        // Final state S^T: the last segment's goes to the pool slot (padding
        // slot 0 is never written); segment 0 of a segmented request hands its
        // end state to segment 1; the first-pass chains leave B and A.
        {
            uint32_t r[SC];
            tmem_ld<SC>(tq + kColS + SC * cs, r);
            tmem_ld_wait();
            auto put = [&](float *xs) {
                if (srow < D) {
#pragma unroll
                    for (int e = 0; e < SC / 4; ++e)
                        *reinterpret_cast<float4 *>(xs + ((SC / 4 * cs + e) * D + srow) * 4) =
                            make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                        __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
                }
            };
            if (truth && seg == nseg - 1 && (nseg == 1 || half)) {
                float *hs = p.state + slot * s0 + h * s1;
                if (slot > 0 && srow < D) {
#pragma unroll
                    for (int e = 0; e < SC; ++e) hs[srow * sv + (SC * cs + e) * sk] = __uint_as_float(r[e]);
                }
            } else if (truth && seg == 0) {
                put(xslot(kSlotStart, 1));
            } else if (!truth) {
                // a full chain ends with its B or A; a half chain's end is its
                // midpoint state (as is a one-chunk segment's)
                if (!half) put(xslot(kind, seg));
                if (half || mid_at == nchunks) put(xslot(kind + 2, seg));
            }
        }
    }
    // After an expired wait: thread 0 waits (bounded, without the shortcut)
    // for the last state update and the last chunk's operand copies before
    // the CTA frees its tensor memory and exits.
    if (*abort_w != 0 && tid == 0 && nchunks > 0) {
        const uint32_t lph = static_cast<uint32_t>((nchunks - 1) & 1);
        mbar_wait(bG4, lph, nullptr);
        mbar_wait(lW, lph, nullptr);
        mbar_wait(lKD, lph, nullptr);
        mbar_wait(lEgl, lph, nullptr);
        if (use_u) {
            const int n0c = (nchunks + 1) / 2, n1c = nchunks / 2;   // copies into U slot 0 and 1
            mbar_wait(lU0, static_cast<uint32_t>((n0c - 1) & 1), nullptr);
            if (n1c > 0) mbar_wait(lU1, static_cast<uint32_t>((n1c - 1) & 1), nullptr);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// Split path, segmented scan, the combine step: one CTA per (request, head)
// with >= 3 segments chains the start states through the first pass's
// segment transfers, S_start[i+1]^T = S_start[i]^T A_i^T + B_i^T for
// i = 1 .. P-2 (S_start[1] is segment 0's end state). Each step is a D x D x D
// split-bf16 mma.sync product with the B term as the accumulator's start; the
// new start state stays in shared memory (bf16 hi/lo) for the next step.
template <int D>
struct CombSmem {
    static constexpr int kSh = 0;                      // S^T hi/lo, swizzled [v][j]
    static constexpr int kSl = kSh + D * D * 2;
    static constexpr int kXh = kSl + D * D * 2;        // A^T hi/lo, swizzled [j][k]
    static constexpr int kXl = kXh + D * D * 2;
    static constexpr int kAlloc = kXl + D * D * 2 + 1024;
};

// fp32 state (exchange layout) in registers: this thread's float4 groups
// q = tid + 512 i of the D x D state (row q % D, columns 4 (q / D) ..).
template <int D>
struct StateRegs {
    static constexpr int N = D * D / 4 / kThreads;
    float4 x[N];
    __device__ __forceinline__ void load(const float *src) {
#pragma unroll
        for (int i = 0; i < N; ++i)
            x[i] = __ldg(reinterpret_cast<const float4 *>(src) + threadIdx.x + kThreads * i);
    }
    // -> bf16 hi/lo swizzled row-major tile in shared memory.
    __device__ __forceinline__ void to_tile(unsigned char *hi, unsigned char *lo) const {
#pragma unroll
        for (int i = 0; i < N; ++i) {
            const int q = threadIdx.x + kThreads * i, row = q % D, c4 = q / D;
            uint32_t h0, h1, l0, l1;
            split2(x[i].x, x[i].y, h0, l0);
            split2(x[i].z, x[i].w, h1, l1);
            const int o = swz<D>(row, 4 * c4) * 2;
            *reinterpret_cast<uint2 *>(hi + o) = make_uint2(h0, h1);
            *reinterpret_cast<uint2 *>(lo + o) = make_uint2(l0, l1);
        }
    }
};

template <int D>
__global__ void __launch_bounds__(kThreads) chunk_combine_kernel(const KdaArgs p, const int32_t *plan,
                                                                float *states) {
    using M = CombSmem<D>;
    constexpr int MT = D / 16;                 // 16-row tiles
    constexpr int WPR = 16 / MT;               // warps per row tile
    constexpr int NC = D / WPR;                // columns per warp
    constexpr int NT = NC / 8;                 // 8-column n-tiles per warp
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    const uint32_t s_base = smem_addr(sm);
    const int req = blockIdx.x / p.head_count, hl = blockIdx.x % p.head_count;
    const PlanView pv(const_cast<int32_t *>(plan), p.num_req, plan[3]);
    const int P = pv.segs()[req];
    if (P < 3) return;
    const int cap = plan[0], sb = pv.sbase()[req];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int mt = warp % MT, n0 = (warp / MT) * NC;
    auto slot = [&](int which, int i) { return state_slot<D>(states, cap, p.head_count, which, i, hl); };
    float acc[NT][4];
    StateRegs<D> xr;
    xr.load(slot(0, sb));
    xr.to_tile(sm + M::kSh, sm + M::kSl);
    xr.load(slot(2, sb));                      // segment 1's A
    for (int i = 1; i + 1 < P; ++i) {
        // slot sb + i - 1 holds segment i's B and A; the result is start state i + 1.
        const float *bt = slot(1, sb + i - 1);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int v = 16 * mt + g + 8 * hf, k = n0 + 8 * nt + 2 * t4;
                const float2 b = __ldg(reinterpret_cast<const float2 *>(bt + ((k >> 2) * D + v) * 4 + (k & 3)));
                acc[nt][2 * hf] = b.x;
                acc[nt][2 * hf + 1] = b.y;
            }
        xr.to_tile(sm + M::kXh, sm + M::kXl);
        __syncthreads();
        if (i + 2 < P) xr.load(slot(2, sb + i));   // the next step's A, in flight during the products
#pragma unroll 2
        for (int ks = 0; ks < D / 16; ++ks) {
            uint32_t ah[4], al[4];
            ldsm_x4(ah, s_base + M::kSh + 2 * lda_a<D>(lane, 16 * mt, 16 * ks));
            ldsm_x4(al, s_base + M::kSl + 2 * lda_a<D>(lane, 16 * mt, 16 * ks));
#pragma unroll
            for (int np = 0; np < NT / 2; ++np) {
                uint32_t bh[4], bl[4];
                ldsm_x4_t(bh, s_base + M::kXh + 2 * lda_b_kn<D>(lane, 16 * ks, n0 + 16 * np));
                ldsm_x4_t(bl, s_base + M::kXl + 2 * lda_b_kn<D>(lane, 16 * ks, n0 + 16 * np));
                mma3(acc[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
                mma3(acc[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
            }
        }
        __syncthreads();
        float *out = slot(0, sb + i);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int v = 16 * mt + g + 8 * hf, k = n0 + 8 * nt + 2 * t4;
                const float x0 = acc[nt][2 * hf], x1 = acc[nt][2 * hf + 1];
                *reinterpret_cast<float2 *>(out + ((k >> 2) * D + v) * 4 + (k & 3)) = make_float2(x0, x1);
                uint32_t hi2, lo2;
                split2(x0, x1, hi2, lo2);
                const int o = swz<D>(v, k) * 2;
                *reinterpret_cast<uint32_t *>(sm + M::kSh + o) = hi2;
                *reinterpret_cast<uint32_t *>(sm + M::kSl + o) = lo2;
            }
        // The next step's A conversion overwrites only the X tiles; its
        // barrier orders these S writes before the next products read them.
    }
}

// The combine on the tensor core (D = 128): the same chain of start states,
// S_start[i+1]^T = S_start[i]^T A_i^T + B_i^T, with S^T in tensor memory
// (fp32 accumulator, and its bf16 hi/lo split as the A operand) and A_i^T as a
// 128-byte-swizzled MN-major B operand in shared memory (rows j, 64-column
// blocks of 128 rows x 128 B). Each step: B_i^T into the accumulator by
// tensor-memory stores, 24 products (8 k-steps x hi.hi + hi.lo + lo.hi), then
// the new start state out to its slot and split for the next step. 256
// threads: warp w reads lanes [32 (w % 4), +32) and columns [64 (w / 4), +64).
struct CombTcSmem {
    static constexpr int D = 128;
    static constexpr int kXh = 0;                        // A^T hi, then lo
    static constexpr int kXl = kXh + D * D * 2;
    static constexpr int kBar = kXl + D * D * 2;
    static constexpr int kAlloc = kBar + 64 + 1024;
    static constexpr uint32_t cS = 0, cSH = 128, cSL = 192;
};

__global__ void __launch_bounds__(256) chunk_combine_tc_kernel(const KdaArgs p, const int32_t *plan, float *states) {
    constexpr int D = 128;
    using M = CombTcSmem;
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    const uint32_t s_base = smem_addr(sm);
    uint64_t *const bar = reinterpret_cast<uint64_t *>(sm + M::kBar);
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(sm + M::kBar + 16);
    const int req = blockIdx.x / p.head_count, hl = blockIdx.x % p.head_count;
    const PlanView pv(const_cast<int32_t *>(plan), p.num_req, plan[3]);
    const int P = pv.segs()[req];
    if (P < 3) return;
    const int cap = plan[0], sb = pv.sbase()[req];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int q4 = warp & 3, ch = warp >> 2;
    const int row = 32 * q4 + lane;
    auto slot = [&](int which, int i) { return state_slot<D>(states, cap, p.head_count, which, i, hl); };

    if (warp == 0) tmem_alloc(tmem_slot, 256);
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    // This thread's 64 columns of a state in the exchange layout: float4 e
    // holds columns 64 ch + 4 e .. + 3 of row `row`.
    auto load_row = [&](const float *src, float4 (&x)[16]) {
#pragma unroll
        for (int e = 0; e < 16; ++e)
            x[e] = __ldg(reinterpret_cast<const float4 *>(src + ((16 * ch + e) * D + row) * 4));
    };
    auto split_row = [&](const float4 (&x)[16]) {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
            split2(x[e].x, x[e].y, hi[2 * e], lo[2 * e]);
            split2(x[e].z, x[e].w, hi[2 * e + 1], lo[2 * e + 1]);
        }
        tmem_st<32>(tq + M::cSH + 32 * ch, hi);
        tmem_st<32>(tq + M::cSL + 32 * ch, lo);
    };
    {
        float4 x[16];
        load_row(slot(0, sb), x);
        split_row(x);
    }
    constexpr uint32_t id = idesc_bf16(128, D, false, true, false);
    for (int i = 1; i + 1 < P; ++i) {
        const float *at = slot(2, sb + i - 1), *bt = slot(1, sb + i - 1);
        if (tid == 0 && i + 2 < P) {
            bulk_prefetch_l2(slot(2, sb + i), D * D * 4);
            bulk_prefetch_l2(slot(1, sb + i), D * D * 4);
        }
        // A_i^T -> swizzled bf16 hi/lo tile: float4 groups q = tid + 256 e
        // (row q % D, columns 4 (q / D) ..).
#pragma unroll 4
        for (int e = 0; e < D * D / 4 / 256; ++e) {
            const int q = tid + 256 * e, j = q % D, k = 4 * (q / D);
            const float4 x = __ldg(reinterpret_cast<const float4 *>(at) + q);
            uint32_t h0, h1, l0, l1;
            split2(x.x, x.y, h0, l0);
            split2(x.z, x.w, h1, l1);
            const int o = ((k >> 6) * (D * 64) + swz<64>(j, k & 63)) * 2;
            *reinterpret_cast<uint2 *>(sm + M::kXh + o) = make_uint2(h0, h1);
            *reinterpret_cast<uint2 *>(sm + M::kXl + o) = make_uint2(l0, l1);
        }
        {
            // B_i^T starts the accumulator.
            float4 x[16];
            load_row(bt, x);
            uint32_t r[32];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    r[4 * e] = __float_as_uint(x[8 * half + e].x);
                    r[4 * e + 1] = __float_as_uint(x[8 * half + e].y);
                    r[4 * e + 2] = __float_as_uint(x[8 * half + e].z);
                    r[4 * e + 3] = __float_as_uint(x[8 * half + e].w);
                }
                tmem_st<32>(tq + M::cS + 64 * ch + 32 * half, r);
            }
        }
        fence_async_smem();
        tmem_st_wait();
        tc_fence_before();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
                const uint32_t ah = tmem + M::cSH + 8 * kk, al = tmem + M::cSL + 8 * kk;
                const uint64_t xh = sdesc_add(sdesc(s_base, D * 128, 1024), M::kXh + kk * 2048);
                const uint64_t xl = sdesc_add(sdesc(s_base, D * 128, 1024), M::kXl + kk * 2048);
                umma_ts(tmem + M::cS, al, xh, id, 1u);
                umma_ts(tmem + M::cS, ah, xl, id, 1u);
                umma_ts(tmem + M::cS, ah, xh, id, 1u);
            }
            umma_commit(bar);
        }
        if (!mbar_wait(bar, static_cast<uint32_t>((i - 1) & 1), p.status) && tid == 0)
            report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
        tc_fence_after();
        {
            // S_start[i+1]^T -> its slot and the next A operand.
            uint32_t r[32];
            float4 x[16];
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                tmem_ld<32>(tq + M::cS + 64 * ch + 32 * half, r);
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    x[8 * half + e] = make_float4(__uint_as_float(r[4 * e]), __uint_as_float(r[4 * e + 1]),
                                                  __uint_as_float(r[4 * e + 2]), __uint_as_float(r[4 * e + 3]));
            }
            float *out = slot(0, sb + i);
#pragma unroll
            for (int e = 0; e < 16; ++e) *reinterpret_cast<float4 *>(out + ((16 * ch + e) * D + row) * 4) = x[e];
            split_row(x);
        }
        // The next step's tile writes and accumulator stores follow this
        // step's completed products (the barrier wait above).
    }
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// Split path, part 3: the outputs, one CTA per (chunk, head) on all SMs. From
// the chunk's record (W, QG, -u^T, Aqk) and the scan's split of the
// chunk-start state S_c: v' = u - W S_c, then o = QG S_c + Aqk v', as
// split-bf16 mma.sync products; the tile leaves by TMA. Recomputing v' here
// keeps the scan's stores to the state alone (an SM stores 32 B per cycle).
template <int D>
struct OutSmem {
    static constexpr int kW = 0;                               // f64 hi/lo [64][D] (token, key)
    static constexpr int kQG = kW + BT * D * 4;                // f64 hi/lo [64][D] (record order: W, QG)
    static constexpr int kU = kQG + BT * D * 4;                // -u^T, record layout
    static constexpr int kAQ = kU + BT * D * 4;                // swizzled hi/lo [64][64] (record order: U, Aqk)
    static constexpr int kS = kAQ + BT * BT * 4;               // ScanOut layout: S hi/lo
    static constexpr int kV = kS + ScanOut<D>::kBytes;         // v' hi/lo, fr layout [D][64] (value, token)
    static constexpr int kO = kW;                              // bf16 [64][D] output staging (W is dead by then)
    static constexpr int kBar = kV + BT * D * 4;
    static constexpr int kAlloc = kBar + 16 + 1024;
    static_assert(Rec<D>::kQG == Rec<D>::kW + BT * D * 4 && Rec<D>::kAQ == Rec<D>::kU + BT * D * 4,
                  "record pieces the output kernel copies together must be adjacent");
    static_assert(kAlloc <= 232448, "output kernel shared memory exceeds the 227 KiB per-CTA limit");
};

template <int D>
__global__ void __launch_bounds__(kThreads) chunk_out_kernel(const KdaArgs p, const __grid_constant__ TmaMaps maps,
                                                            const uint8_t *rec, const uint8_t *sout,
                                                            const int32_t *cbase) {
    using M = OutSmem<D>;
    using R = Rec<D>;
    using SO = ScanOut<D>;
    constexpr int KS = D / 16;
    constexpr int NT = D / 32;                 // 8-column n-tiles per warp
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    const uint32_t s_base = smem_addr(sm);
    uint64_t *const bar = reinterpret_cast<uint64_t *>(sm + M::kBar);
    __nv_bfloat16 *const Ost = reinterpret_cast<__nv_bfloat16 *>(sm + M::kO);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g = lane >> 2, t4 = lane & 3;
    const int H = p.num_heads;
    const int hl = blockIdx.x % p.head_count, h = p.head_begin + hl;
    const int sl = blockIdx.x / p.head_count;
    int req = 0;
    while (req < p.num_req && cbase[req + 1] <= sl) ++req;
    if (req >= p.num_req) return;
    const int c = sl - cbase[req];
    const int64_t bos = load_index(p.cu_seqlens, p.index_bytes[1], req);
    const int64_t eos = load_index(p.cu_seqlens, p.index_bytes[1], req + 1);
    const int64_t slot = load_index(p.indices, p.index_bytes[0], req);
    if (bos < 0 || eos < bos || eos > p.num_tokens || slot < 0 || slot >= p.num_slots) return;   // reported by the scan
    const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
    const int n = static_cast<int>(eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT));
    const int64_t rix = static_cast<int64_t>(sl) * p.head_count + hl;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        const uint8_t *r = rec + rix * R::kBytes;
        mbar_arrive_expect_tx(bar, 2 * BT * D * 4 + BT * D * 4 + BT * BT * 4 + SO::kBytes);
        bulk_g2s(sm + M::kW, r + R::kW, 2 * BT * D * 4, bar);                  // W, QG
        bulk_g2s(sm + M::kU, r + R::kU, BT * D * 4 + BT * BT * 4, bar);        // -u^T, Aqk
        bulk_g2s(sm + M::kS, sout + rix * SO::kBytes, SO::kBytes, bar);
    }
    __syncthreads();
    if (!mbar_wait(bar, 0, p.status) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);

    // Warp w: tokens [16 (w % 4), +16), values [(w / 4) D/4, +D/4).
    const int mt = warp & 3, v0 = (warp >> 2) * (D / 4);
    float acc[NT][4] = {}, wsv[NT][4] = {};
    const uint32_t sh = s_base + M::kS + SO::kSH, slo = s_base + M::kS + SO::kSL;
    const uint32_t vh = s_base + M::kV, vlo = s_base + M::kV + D * BT * 2;
#pragma unroll 2
    for (int ks = 0; ks < KS; ++ks) {   // QG S_c and W S_c: K = keys, one pass over the S fragments
        uint32_t ah[4], al[4], wh[4], wl[4];
        ldsm_x4(ah, s_base + M::kQG + 2 * fa_a(lane, 16 * mt, 16 * ks));
        ldsm_x4(al, s_base + M::kQG + BT * D * 2 + 2 * fa_a(lane, 16 * mt, 16 * ks));
        ldsm_x4(wh, s_base + M::kW + 2 * fa_a(lane, 16 * mt, 16 * ks));
        ldsm_x4(wl, s_base + M::kW + BT * D * 2 + 2 * fa_a(lane, 16 * mt, 16 * ks));
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            const int q = lane >> 3, r = lane & 7;
            const uint32_t ob = 2 * fr<D>(v0 + 16 * np + r + ((q >> 1) << 3), 16 * ks + ((q & 1) << 3));
            uint32_t bh[4], bl[4];
            ldsm_x4(bh, sh + ob);
            ldsm_x4(bl, slo + ob);
            mma3(acc[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
            mma3(acc[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
            mma3(wsv[2 * np], wh, wl, bh[0], bh[1], bl[0], bl[1]);
            mma3(wsv[2 * np + 1], wh, wl, bh[2], bh[3], bl[2], bl[3]);
        }
    }
    {
        // v' = -(-u + W S_c) -> bf16 hi/lo at (value, token) for Aqk v'.
        const float *us = reinterpret_cast<const float *>(sm + M::kU);
        uint16_t *vph = reinterpret_cast<uint16_t *>(sm + M::kV);
        uint16_t *vpl = vph + D * BT;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int t = 16 * mt + g + 8 * hf, v = v0 + 8 * nt + 2 * t4 + e;
                    const float x = -(us[((t >> 2) * D + v) * 4 + (t & 3)] + wsv[nt][2 * hf + e]);
                    uint16_t xh, xl;
                    split1(x, xh, xl);
                    vph[fr<D>(v, t)] = xh;
                    vpl[fr<D>(v, t)] = xl;
                }
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {    // Aqk v': K = tokens
        uint32_t ah[4], al[4];
        ldsm_x4(ah, s_base + M::kAQ + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
        ldsm_x4(al, s_base + M::kAQ + BT * BT * 2 + 2 * lda_a<BT>(lane, 16 * mt, 16 * ks));
#pragma unroll
        for (int np = 0; np < NT / 2; ++np) {
            const int q = lane >> 3, r = lane & 7;
            const uint32_t ob = 2 * fr<D>(v0 + 16 * np + r + ((q >> 1) << 3), 16 * ks + ((q & 1) << 3));
            uint32_t bh[4], bl[4];
            ldsm_x4(bh, vh + ob);
            ldsm_x4(bl, vlo + ob);
            mma3(acc[2 * np], ah, al, bh[0], bh[1], bl[0], bl[1]);
            mma3(acc[2 * np + 1], ah, al, bh[2], bh[3], bl[2], bl[3]);
        }
    }
    if (p.out_fp32) {
        float *o = static_cast<float *>(p.out);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int t = 16 * mt + g + 8 * hf, v = v0 + 8 * nt + 2 * t4;
                if (t < n) {
                    float *row = o + ((t0 + t) * H + h) * D + v;
                    row[0] = acc[nt][2 * hf];
                    row[1] = acc[nt][2 * hf + 1];
                }
            }
        return;
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
            const int t = 16 * mt + g + 8 * hf, v = v0 + 8 * nt + 2 * t4;
            *reinterpret_cast<uint32_t *>(Ost + t * D + v) = pack_bf16(acc[nt][2 * hf], acc[nt][2 * hf + 1]);
        }
    fence_async_smem();
    __syncthreads();
    if (tid == 0) {
        if (n == BT) {
            tma_store_3d(&maps.o, Ost, 0, h, static_cast<int>(t0));
        } else {
            __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + (t0 * H + h) * D;
            for (int rw = 0; rw < n; ++rw) bulk_s2g(o + static_cast<int64_t>(rw) * H * D, Ost + rw * D, D * 2);
        }
        bulk_commit();
        bulk_wait_read();
    }
}

// Split path, part 3 on the tensor core (D = 128): the same outputs as
// chunk_out_kernel, o^T = S_c^T QG^T + v'^T Aqk^T with -v'^T = -u^T + S_c^T W^T,
// as tcgen05 products with value rows on the 128 tensor-memory lanes. The
// scan's state split is already the no-swizzle K-major operand layout (8-row
// x 16-byte core matrices, +128 B along the value rows, +2 KB along the keys),
// so it feeds the tensor core straight from its bulk copy; W, QG and Aqk are
// the record's 128-byte-swizzled tiles. -u^T goes from the record into the
// v' accumulator by tensor-memory stores. 256 threads: warp w reads lanes
// [32 (w % 4), +32) and token columns [32 (w / 4), +32).
struct OutTcSmem {
    static constexpr int D = 128;
    static constexpr int kS = 0;                             // ScanOut: S hi, S lo (fr layout)
    static constexpr int kW = ScanOut<D>::kBytes;            // W hi/lo, then QG hi/lo (record order)
    static constexpr int kQG = kW + BT * D * 4;
    static constexpr int kAQ = kQG + BT * D * 4;             // Aqk hi/lo, swizzled [64][64]
    static constexpr int kO = kAQ + BT * BT * 4;             // bf16 [64][D] output staging
    static constexpr int kBar = kO + BT * D * 2;             // 3 mbarriers + tensor-memory base slot
    static constexpr int kAlloc = kBar + 64 + 1024;
    // Tensor-memory columns (256 allocated).
    static constexpr uint32_t cNU = 0, cO = 64, cVH = 128, cVL = 160;
    static_assert(Rec<D>::kQG == Rec<D>::kW + BT * D * 4, "W and QG are one copy");
    static_assert((kW & 1023) == 0 && (kQG & 1023) == 0 && (kAQ & 1023) == 0, "swizzled tiles need 1 KB alignment");
};

__global__ void __launch_bounds__(256) chunk_out_tc_kernel(const KdaArgs p, const __grid_constant__ TmaMaps maps,
                                                          const uint8_t *rec, const uint8_t *sout,
                                                          const int32_t *cbase) {
    constexpr int D = 128;
    using M = OutTcSmem;
    using R = Rec<D>;
    using SO = ScanOut<D>;
    extern __shared__ __align__(1024) unsigned char sm_raw[];
    unsigned char *const sm = sm_raw + ((1024u - (smem_addr(sm_raw) & 1023u)) & 1023u);
    const uint32_t s_base = smem_addr(sm);
    uint64_t *const bars = reinterpret_cast<uint64_t *>(sm + M::kBar);   // 0 operands, 1 W S, 2 all products
    uint32_t *const tmem_slot = reinterpret_cast<uint32_t *>(sm + M::kBar + 32);
    __nv_bfloat16 *const Ost = reinterpret_cast<__nv_bfloat16 *>(sm + M::kO);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int q4 = warp & 3, ch = warp >> 2;
    const int row = 32 * q4 + lane;                      // value row
    const int H = p.num_heads;
    const int hl = blockIdx.x % p.head_count, h = p.head_begin + hl;
    const int sl = blockIdx.x / p.head_count;
    int req = 0;
    while (req < p.num_req && cbase[req + 1] <= sl) ++req;
    if (req >= p.num_req) return;
    const int c = sl - cbase[req];
    const int64_t bos = load_index(p.cu_seqlens, p.index_bytes[1], req);
    const int64_t eos = load_index(p.cu_seqlens, p.index_bytes[1], req + 1);
    const int64_t slot = load_index(p.indices, p.index_bytes[0], req);
    if (bos < 0 || eos < bos || eos > p.num_tokens || slot < 0 || slot >= p.num_slots) return;   // reported by the scan
    const int64_t t0 = bos + static_cast<int64_t>(c) * BT;
    const int n = static_cast<int>(eos - t0 < BT ? eos - t0 : static_cast<int64_t>(BT));
    const int64_t rix = static_cast<int64_t>(sl) * p.head_count + hl;   // == blockIdx.x
    const uint8_t *const r = rec + rix * R::kBytes;

    if (warp == 0) tmem_alloc(tmem_slot, 256);
    if (tid == 0) {
#pragma unroll
        for (int i = 0; i < 3; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(&bars[0], SO::kBytes + 2 * BT * D * 4 + BT * BT * 4);
        bulk_g2s(sm + M::kS, sout + rix * SO::kBytes, SO::kBytes, &bars[0]);
        bulk_g2s(sm + M::kW, r + R::kW, 2 * BT * D * 4, &bars[0]);
        bulk_g2s(sm + M::kAQ, r + R::kAQ, BT * BT * 4, &bars[0]);
        // The CTA one wave later (block + SM count; its record index is its
        // block index) finds its operands in L2.
        uint32_t nsm;
        asm("mov.u32 %0, %%nsmid;" : "=r"(nsm));
        const int64_t nb = static_cast<int64_t>(blockIdx.x) + nsm;
        if (nb < static_cast<int64_t>(gridDim.x)) {
            const uint8_t *r2 = rec + nb * R::kBytes;
            bulk_prefetch_l2(sout + nb * SO::kBytes, SO::kBytes);
            bulk_prefetch_l2(r2 + R::kW, 2 * BT * D * 4);
            bulk_prefetch_l2(r2 + R::kU, BT * D * 4 + BT * BT * 4);
        }
    }
    // -u^T of value row `row`, tokens [32 ch, +32): float (t, v) of the record
    // at ((t / 4) D + v) * 4 + t % 4, so a warp's float4 loads are 512
    // contiguous bytes.
    uint32_t x[32];
    {
        const float *us = reinterpret_cast<const float *>(r + R::kU);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float4 u4 = __ldg(reinterpret_cast<const float4 *>(us + ((8 * ch + k) * D + row) * 4));
            x[4 * k] = __float_as_uint(u4.x);
            x[4 * k + 1] = __float_as_uint(u4.y);
            x[4 * k + 2] = __float_as_uint(u4.z);
            x[4 * k + 3] = __float_as_uint(u4.w);
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t tq = tmem + (static_cast<uint32_t>(32 * q4) << 16);
    tmem_st<32>(tq + M::cNU + 32 * ch, x);
    tmem_st_wait();
    tc_fence_before();
    __syncthreads();   // the v' accumulator holds -u^T
    constexpr uint32_t id_n64 = idesc_bf16(128, 64, false, false, false);
    if (tid == 0) {
        tc_fence_after();
        if (!mbar_wait(&bars[0], 0, p.status)) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
        // -v'^T = -u^T + S^T W^T, then o^T = S^T QG^T (split-bf16: hi.hi + hi.lo + lo.hi).
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ah = sdesc_noswz(s_base + M::kS + SO::kSH + kk * 4096, 2048, 128);
            const uint64_t al = sdesc_noswz(s_base + M::kS + SO::kSL + kk * 4096, 2048, 128);
            const uint32_t off = (kk >> 2) * 8192 + (kk & 3) * 32;
            const uint64_t wh = sdesc_add(sdesc(s_base, 16, 1024), M::kW + off);
            const uint64_t wl = sdesc_add(sdesc(s_base, 16, 1024), M::kW + BT * D * 2 + off);
            umma_ss(tmem + M::cNU, al, wh, id_n64, 1u);
            umma_ss(tmem + M::cNU, ah, wl, id_n64, 1u);
            umma_ss(tmem + M::cNU, ah, wh, id_n64, 1u);
        }
        umma_commit(&bars[1]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
            const uint64_t ah = sdesc_noswz(s_base + M::kS + SO::kSH + kk * 4096, 2048, 128);
            const uint64_t al = sdesc_noswz(s_base + M::kS + SO::kSL + kk * 4096, 2048, 128);
            const uint32_t off = (kk >> 2) * 8192 + (kk & 3) * 32;
            const uint64_t qh = sdesc_add(sdesc(s_base, 16, 1024), M::kQG + off);
            const uint64_t ql = sdesc_add(sdesc(s_base, 16, 1024), M::kQG + BT * D * 2 + off);
            umma_ss(tmem + M::cO, al, qh, id_n64, kk > 0 ? 1u : 0u);
            umma_ss(tmem + M::cO, ah, ql, id_n64, 1u);
            umma_ss(tmem + M::cO, ah, qh, id_n64, 1u);
        }
    }
    // -v'^T (fp32) -> v'^T hi/lo A operand, this warp's 32 token columns.
    if (!mbar_wait(&bars[1], 0, p.status) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
    tc_fence_after();
    {
        uint32_t hi[16], lo[16];
        tmem_ld<32>(tq + M::cNU + 32 * ch, x);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e)
            split2(-__uint_as_float(x[2 * e]), -__uint_as_float(x[2 * e + 1]), hi[e], lo[e]);
        tmem_st<16>(tq + M::cVH + 16 * ch, hi);
        tmem_st<16>(tq + M::cVL + 16 * ch, lo);
        tmem_st_wait();
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0) {
        tc_fence_after();
        // o^T += v'^T Aqk^T (K = the chunk's tokens).
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
            const uint32_t ah = tmem + M::cVH + 8 * kk, al = tmem + M::cVL + 8 * kk;
            const uint64_t qh = sdesc_add(sdesc(s_base, 16, 1024), M::kAQ + kk * 32);
            const uint64_t ql = sdesc_add(sdesc(s_base, 16, 1024), M::kAQ + BT * BT * 2 + kk * 32);
            umma_ts(tmem + M::cO, al, qh, id_n64, 1u);
            umma_ts(tmem + M::cO, ah, ql, id_n64, 1u);
            umma_ts(tmem + M::cO, ah, qh, id_n64, 1u);
        }
        umma_commit(&bars[2]);
    }
    if (!mbar_wait(&bars[2], 0, p.status) && tid == 0) report(p.status, KDA_DEVICE_ERR_WAIT_TIMEOUT);
    tc_fence_after();
    tmem_ld<32>(tq + M::cO + 32 * ch, x);
    tmem_ld_wait();
    if (p.out_fp32) {
        float *o = static_cast<float *>(p.out);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
            const int t = 32 * ch + e;
            if (t < n) o[((t0 + t) * H + h) * D + row] = __uint_as_float(x[e]);
        }
    } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) Ost[(32 * ch + e) * D + row] = __float2bfloat16_rn(__uint_as_float(x[e]));
        fence_async_smem();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
    if (tid == 0 && !p.out_fp32) {
        if (n == BT) {
            tma_store_3d(&maps.o, Ost, 0, h, static_cast<int>(t0));
        } else {
            __nv_bfloat16 *o = static_cast<__nv_bfloat16 *>(p.out) + (t0 * H + h) * D;
            for (int rw = 0; rw < n; ++rw) bulk_s2g(o + static_cast<int64_t>(rw) * H * D, Ost + rw * D, D * 2);
        }
        bulk_commit();
        bulk_wait_read();
    }
}

// Split-path plan, one thread per request (num_req <= 1024): the chunk slot
// offsets cbase[r] (chunks of requests < r, num_req + 1 entries) and the
// segmentation. The segment length is the shortest (>= kMinSegChunks) whose
// first pass fits `budget` CTAs per head, so that pass runs in one wave.
__global__ void __launch_bounds__(1024) plan_kernel(const KdaArgs p, int32_t *cbase, int32_t *plan, int budget,
                                                   int task_cap, int slot_cap) {
    __shared__ int32_t tmp[32];
    const int r = threadIdx.x;
    const bool live = r < p.num_req;
    int n = 0;
    if (live) {
        const int64_t len = load_index(p.cu_seqlens, p.index_bytes[1], r + 1) -
                            load_index(p.cu_seqlens, p.index_bytes[1], r);
        n = static_cast<int>(len > 0 ? (len + BT - 1) / BT : 0);
    }
    int total;
    const int cb = block_scan(n, tmp, total);
    if (live) cbase[r] = cb;
    if (r == 0) cbase[p.num_req] = total;
    auto segs = [&](int L) { return n <= L ? 1 : max(3, (n + L - 1) / L); };
    // First-pass CTAs per request: segment 0, two chains per middle segment,
    // two half chains for the last (the rescan needs 2 (P - 1), fewer).
    auto cost = [&](int L) {
        const int P = segs(L);
        return live ? (P == 1 ? 1 : 2 * P - 1) : 0;
    };
    const int maxn = block_max(n, tmp);
    int hi = max(maxn, kMinSegChunks), lo = kMinSegChunks;
    int t;
    block_scan(cost(lo), tmp, t);
    if (t > budget) {
        // Binary search for the shortest segment whose first pass fits.
        while (lo < hi) {
            const int mid = (lo + hi) / 2;
            block_scan(cost(mid), tmp, t);
            if (t <= budget) hi = mid;
            else lo = mid + 1;
        }
    } else {
        hi = lo;
    }
    const int L = hi;
    const PlanView pv(plan, p.num_req, task_cap);
    const int P = live ? segs(L) : 0;
    int na, nc;
    const int oa = block_scan(live ? (P == 1 ? 1 : 2 * P - 1) : 0, tmp, na);
    const int oc = block_scan(P >= 3 ? 2 * (P - 1) : 0, tmp, nc);
    const int os = block_scan(P >= 3 ? P - 1 : 0, tmp, total);   // state slots
    if (live) {
        pv.segs()[r] = P;
        pv.seglen()[r] = (n + P - 1) / P;
        pv.sbase()[r] = os;
        int32_t *ta = pv.tasks(0), *tc = pv.tasks(1);
        ta[oa] = task_word(r, kTaskTrue, 0);
        for (int sg = 1; sg < P && P >= 3; ++sg) {
            const int half = sg == P - 1 ? 1 : 0;
            ta[oa + 2 * sg - 1] = task_word(r, kTaskZero, sg, half);
            ta[oa + 2 * sg] = task_word(r, kTaskIdent, sg, half);
            tc[oc + 2 * (sg - 1)] = task_word(r, kTaskTrue, sg, 0);
            tc[oc + 2 * (sg - 1) + 1] = task_word(r, kTaskTrue, sg, 1);
        }
    }
    if (r == 0) {
        plan[0] = slot_cap;
        plan[1] = na;
        plan[2] = nc;
        plan[3] = task_cap;
    }
}

}  // namespace chunk

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

static bool chunk_aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

static size_t order_bytes(int32_t num_req) {
    return (static_cast<size_t>(num_req > 0 ? num_req : 1) * sizeof(int32_t) + 255) / 256 * 256;
}

// cuTensorMapEncodeTiled, resolved once through the runtime's driver entry
// point (the library links the static runtime, not libcuda).
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return static_cast<EncodeTiledFn>(nullptr);
        return reinterpret_cast<EncodeTiledFn>(ptr);
    }();
    return fn;
}

// A [T][H][D] tensor seen as (x = column, y = head, z = token), box of
// `box_x` columns x 1 head x 64 tokens. Tokens past T read as zero.
static bool encode_rows(CUtensorMap *map, const void *base, CUtensorMapDataType type, int elem_bytes, int D,
                        int H, int64_t T, int box_x, CUtensorMapSwizzle swizzle) {
    const EncodeTiledFn fn = encode_tiled();
    if (fn == nullptr) return false;
    const cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                                static_cast<cuuint64_t>(T > 0 ? T : 1)};
    const cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * elem_bytes,
                                   static_cast<cuuint64_t>(D) * elem_bytes * H};
    const cuuint32_t box[3] = {static_cast<cuuint32_t>(box_x), 1u, static_cast<cuuint32_t>(chunk::BT)};
    const cuuint32_t estr[3] = {1u, 1u, 1u};
    return fn(map, type, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

static bool encode_maps(chunk::TmaMaps &maps, const KdaArgs *a, int D, bool raw) {
    const int H = a->num_heads;
    const int64_t T = a->num_tokens;
    return encode_rows(&maps.q, a->q, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, H, T, D, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           encode_rows(&maps.k, a->k, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, H, T, D, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           encode_rows(&maps.g, raw ? a->a : a->g,
                       raw ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, raw ? 2 : 4, D, H,
                       T, D, CU_TENSOR_MAP_SWIZZLE_NONE) &&
           encode_rows(&maps.v, a->v, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, H, T, 64, CU_TENSOR_MAP_SWIZZLE_128B) &&
           encode_rows(&maps.o, a->out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, D, H, T, D, CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Opt a kernel into the chunk kernels' dynamic shared memory once per device.
template <typename K>
static bool opt_in(K kernel, bool (&done)[64], int bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    dev = (dev >= 0 && dev < 64) ? dev : 0;
    if (!done[dev]) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
            return false;
        done[dev] = true;
    }
    return true;
}

template <int D, int MODE>
static int launch_chunk(const KdaArgs *a, int32_t *order, cudaStream_t st, int32_t skip_hi) {
    using L = chunk::Smem<D>;
    chunk::TmaMaps maps;
    if (!encode_maps(maps, a, D, MODE == KDA_GATE_RAW)) return KDA_ERR_LAUNCH;
    static bool opted[64];
    if (!opt_in(chunk::chunk_kernel<D, MODE, false>, opted, L::kAlloc)) return KDA_ERR_LAUNCH;
    if (order != nullptr) chunk::order_kernel<<<1, 1024, 0, st>>>(*a, order);
    const int64_t grid = static_cast<int64_t>(a->num_req) * a->head_count;
    chunk::chunk_kernel<D, MODE, false><<<static_cast<unsigned>(grid), chunk::kThreads + 32, L::kAlloc, st>>>(
        *a, order, maps, nullptr, nullptr, nullptr, skip_hi);
    return KDA_OK;
}

// ---- Split path: which batches use it, and its workspace ----
//
// The fused kernel runs one CTA per (sequence, head) chain through every
// phase of every chunk; that fills the GPU when there are many chains. With
// few chains (a long context over a few heads) most SMs would idle, so the
// split path first computes every chunk's intra-chunk operands with one CTA
// per (chunk, head) on all SMs, then runs only the serial scan per chain.

static int sm_count() {
    static int count[64];
    int dev = 0;
    cudaGetDevice(&dev);
    dev = (dev >= 0 && dev < 64) ? dev : 0;
    if (count[dev] == 0) {
        int c = 0;
        cudaDeviceGetAttribute(&c, cudaDevAttrMultiProcessorCount, dev);
        count[dev] = c > 0 ? c : 1;
    }
    return count[dev];
}

static bool split_ok(int32_t num_req) { return num_req > 0 && num_req <= 1024; }

// Longest request the fused path hands to the token recurrence.
constexpr int32_t kShortLen = 16;

// The library's own choice: the split path when the (sequence, head) chains
// fill at most half the SMs and the sequences average >= 8 chunks.
static bool want_split(int32_t num_req, int32_t heads, int32_t num_tokens) {
    const int64_t chains = static_cast<int64_t>(num_req) * heads;
    return split_ok(num_req) && chains * 2 <= sm_count() &&
           static_cast<int64_t>(num_tokens) >= static_cast<int64_t>(num_req) * chunk::BT * 8;
}

static size_t a256(size_t x) { return (x + 255) / 256 * 256; }

// Split-path workspace: chunk offsets, the segmentation plan, the per-chunk
// records, the tracked-prefix records, the state splits for the output
// kernel, and the segment-boundary states (start, B, A) of the segmented scan.
// The first pass gets `budget` CTAs per head, so that it runs in one wave.
struct SplitLayout {
    size_t cbase, plan, rec, trec, sout, states, total;
    int budget, task_cap, slot_cap;
};
static SplitLayout split_layout(int32_t num_req, int32_t num_tokens, int32_t heads, int32_t D) {
    const size_t slots = static_cast<size_t>(num_tokens) / chunk::BT + static_cast<size_t>(num_req);
    const size_t rb = D == 64 ? chunk::Rec<64>::kBytes : chunk::Rec<128>::kBytes;
    const size_t tb = D == 64 ? chunk::Rec<64>::tBytes : chunk::Rec<128>::tBytes;
    const size_t ob = D == 64 ? chunk::ScanOut<64>::kBytes : chunk::ScanOut<128>::kBytes;
    SplitLayout l;
    l.budget = std::max(1, sm_count() / std::max(1, static_cast<int>(heads)));
    l.task_cap = std::max(l.budget, static_cast<int>(num_req));
    l.slot_cap = l.budget;
    l.cbase = 0;
    l.plan = a256((static_cast<size_t>(num_req) + 1) * sizeof(int32_t));
    l.rec = l.plan + a256(chunk::PlanView::words(num_req, l.task_cap) * sizeof(int32_t));
    l.trec = l.rec + slots * static_cast<size_t>(heads) * rb;
    l.sout = l.trec + static_cast<size_t>(num_req) * static_cast<size_t>(heads) * tb;
    l.states = l.sout + slots * static_cast<size_t>(heads) * ob;
    l.total = l.states + static_cast<size_t>(chunk::kSlotKinds) * static_cast<size_t>(l.slot_cap) *
                             static_cast<size_t>(heads) * D * D * sizeof(float);
    return l;
}

// `ev` (measurement only, else null): six events recorded on the stream before
// the plan and after prep, the scan's first pass, the combine, the rescan and
// the outputs.
template <int D, int MODE>
static int launch_chunk_split(const KdaArgs *a, uint8_t *ws, cudaStream_t st, cudaEvent_t const *ev = nullptr) {
    using L = chunk::Smem<D>;
    chunk::TmaMaps maps;
    if (!encode_maps(maps, a, D, MODE == KDA_GATE_RAW)) return KDA_ERR_LAUNCH;
    static bool opted_prep[64], opted_scan[64], opted_comb[64], opted_comb_tc[64], opted_out[64], opted_out_tc[64];
    if (!opt_in(chunk::chunk_kernel<D, MODE, true>, opted_prep, L::kAlloc) ||
        !opt_in(chunk::chunk_scan_kernel<D>, opted_scan, L::kAlloc) ||
        !opt_in(chunk::chunk_combine_kernel<D>, opted_comb, chunk::CombSmem<D>::kAlloc) ||
        !opt_in(chunk::chunk_out_kernel<D>, opted_out, chunk::OutSmem<D>::kAlloc) ||
        (D == 128 && !opt_in(chunk::chunk_out_tc_kernel, opted_out_tc, chunk::OutTcSmem::kAlloc)) ||
        (D == 128 && !opt_in(chunk::chunk_combine_tc_kernel, opted_comb_tc, chunk::CombTcSmem::kAlloc)))
        return KDA_ERR_LAUNCH;
    const SplitLayout lay = split_layout(a->num_req, a->num_tokens, a->head_count, D);
    int32_t *cbase = reinterpret_cast<int32_t *>(ws + lay.cbase);
    int32_t *plan = reinterpret_cast<int32_t *>(ws + lay.plan);
    uint8_t *rec = ws + lay.rec, *trec = ws + lay.trec, *sout = ws + lay.sout;
    float *states = reinterpret_cast<float *>(ws + lay.states);
    auto mark = [&](int i) {
        if (ev != nullptr) cudaEventRecord(ev[i], st);
    };
    mark(0);
    chunk::plan_kernel<<<1, 1024, 0, st>>>(*a, cbase, plan, lay.budget, lay.task_cap, lay.slot_cap);
    const int64_t slots = static_cast<int64_t>(a->num_tokens) / chunk::BT + a->num_req;
    chunk::chunk_kernel<D, MODE, true><<<static_cast<unsigned>(slots * a->head_count), chunk::kThreads + 32,
                                         L::kAlloc, st>>>(*a, nullptr, maps, rec, trec, cbase, 0);
    mark(1);
    // Segmented scan: first pass, combine, rescan (CTAs past a phase's task
    // count exit at once).
    const unsigned scan_grid = static_cast<unsigned>(static_cast<int64_t>(lay.task_cap) * a->head_count);
    chunk::chunk_scan_kernel<D><<<scan_grid, chunk::kThreads + 32, L::kAlloc, st>>>(*a, plan, 0, maps, rec, trec,
                                                                                 cbase, sout, states);
    mark(2);
    if constexpr (D == 128) {
        chunk::chunk_combine_tc_kernel<<<static_cast<unsigned>(static_cast<int64_t>(a->num_req) * a->head_count), 256,
                                         chunk::CombTcSmem::kAlloc, st>>>(*a, plan, states);
    } else {
        chunk::chunk_combine_kernel<D><<<static_cast<unsigned>(static_cast<int64_t>(a->num_req) * a->head_count),
                                         chunk::kThreads, chunk::CombSmem<D>::kAlloc, st>>>(*a, plan, states);
    }
    mark(3);
    chunk::chunk_scan_kernel<D><<<scan_grid, chunk::kThreads + 32, L::kAlloc, st>>>(*a, plan, 1, maps, rec, trec,
                                                                                 cbase, sout, states);
    mark(4);
    if constexpr (D == 128) {
        chunk::chunk_out_tc_kernel<<<static_cast<unsigned>(slots * a->head_count), 256, chunk::OutTcSmem::kAlloc,
                                     st>>>(*a, maps, rec, sout, cbase);
    } else {
        chunk::chunk_out_kernel<D><<<static_cast<unsigned>(slots * a->head_count), chunk::kThreads,
                                     chunk::OutSmem<D>::kAlloc, st>>>(*a, maps, rec, sout, cbase);
    }
    mark(5);
    return KDA_OK;
}

}  // namespace kda

namespace kda {
// Workspace bytes of a chunk launch that takes `path` (KdaChunkPath).
static size_t chunk_ws_bytes(int32_t num_req, int32_t num_tokens, int32_t heads, int32_t head_dim, int path) {
    if (num_req <= 0) return 0;
    const bool dims_ok = (head_dim == 64 || head_dim == 128) && num_tokens >= 0 && heads > 0;
    const bool split = path == KDA_CHUNK_SPLIT ? split_ok(num_req)
                                               : path == KDA_CHUNK_AUTO && want_split(num_req, heads, num_tokens);
    if (dims_ok && split) return split_layout(num_req, num_tokens, heads, head_dim).total;
    return num_req <= 1024 ? order_bytes(num_req) : 0;
}
}  // namespace kda

extern "C" size_t kda_chunk_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads,
                                            int32_t head_dim) {
    return kda::chunk_ws_bytes(num_req, num_tokens, num_heads, head_dim, KDA_CHUNK_AUTO);
}

extern "C" size_t kda_chunk_path_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads,
                                                 int32_t head_dim, int32_t path) {
    if (path != KDA_CHUNK_AUTO && path != KDA_CHUNK_FUSED && path != KDA_CHUNK_SPLIT) return 0;
    return kda::chunk_ws_bytes(num_req, num_tokens, num_heads, head_dim, path);
}

namespace kda {
// Argument checks of kda_chunk_launch (KDA_OK, or the status to return;
// *empty = nothing to launch).
static int chunk_check(const KdaArgs *args, bool *empty) {
    *empty = false;
    if (args == nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->intermediate != nullptr) return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_PREPARED) return KDA_ERR_UNSUPPORTED;
    if (args->head_dim != 64 && args->head_dim != 128) return KDA_ERR_UNSUPPORTED;
    if (args->num_req < 0 || args->num_tokens < 0 || args->num_heads <= 0 || args->head_begin < 0 ||
        args->head_count < 0 || args->head_begin + args->head_count > args->num_heads)
        return KDA_ERR_INVALID_ARGUMENT;
    for (int i = 0; i < 4; ++i)
        if (args->index_bytes[i] != 4 && args->index_bytes[i] != 8) return KDA_ERR_INVALID_ARGUMENT;
    if (args->num_req == 0 || args->head_count == 0) {
        *empty = true;
        return KDA_OK;
    }
    if (args->state == nullptr || args->num_slots <= 0 || args->indices == nullptr || args->cu_seqlens == nullptr ||
        args->out == nullptr || args->q == nullptr || args->k == nullptr || args->v == nullptr)
        return KDA_ERR_INVALID_ARGUMENT;
    if ((args->track_indices == nullptr) != (args->track_lens == nullptr)) return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_RAW &&
        (args->a == nullptr || args->b == nullptr || args->A_log == nullptr || args->dt_bias == nullptr))
        return KDA_ERR_INVALID_ARGUMENT;
    if (args->gate_mode == KDA_GATE_LOG && (args->g == nullptr || args->beta == nullptr))
        return KDA_ERR_INVALID_ARGUMENT;
    // Tensor-map bases must be 16-byte aligned; the row strides (D elements)
    // are multiples of 16 bytes for both head dims.
    const void *rows[] = {args->q, args->k, args->v, args->gate_mode == KDA_GATE_RAW ? args->a : args->g, args->out};
    for (const void *ptr : rows)
        if (!chunk_aligned16(ptr)) return KDA_ERR_ALIGNMENT;
    return KDA_OK;
}
}  // namespace kda

// Measurement entry point (no counterpart in the reference): the split path
// of kda_chunk_launch with `events` (6 cudaEvent_t, created by the caller)
// recorded on the stream before the plan and after prep, the scan's first
// pass, the combine, the rescan and the outputs. KDA_ERR_UNSUPPORTED when the
// batch would not take the split path, KDA_ERR_WORKSPACE when the workspace
// does not hold it.
extern "C" int kda_chunk_launch_phases(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream,
                                       void *const *events, int num_events) {
    bool empty = false;
    const int chk = kda::chunk_check(args, &empty);
    if (chk != KDA_OK) return chk;
    if (events == nullptr || num_events != 6) return KDA_ERR_INVALID_ARGUMENT;
    if (empty || !kda::want_split(args->num_req, args->head_count, args->num_tokens)) return KDA_ERR_UNSUPPORTED;
    if (workspace == nullptr || (reinterpret_cast<uintptr_t>(workspace) & 255u) != 0 ||
        workspace_bytes < kda::split_layout(args->num_req, args->num_tokens, args->head_count, args->head_dim).total)
        return KDA_ERR_WORKSPACE;
    cudaEvent_t ev[6];
    for (int i = 0; i < 6; ++i) ev[i] = static_cast<cudaEvent_t>(events[i]);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t *ws = static_cast<uint8_t *>(workspace);
    int rc;
    if (args->head_dim == 128)
        rc = args->gate_mode == KDA_GATE_RAW ? kda::launch_chunk_split<128, KDA_GATE_RAW>(args, ws, st, ev)
                                             : kda::launch_chunk_split<128, KDA_GATE_LOG>(args, ws, st, ev);
    else
        rc = args->gate_mode == KDA_GATE_RAW ? kda::launch_chunk_split<64, KDA_GATE_RAW>(args, ws, st, ev)
                                             : kda::launch_chunk_split<64, KDA_GATE_LOG>(args, ws, st, ev);
    if (rc != KDA_OK) return rc;
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}

namespace kda {
// kda_chunk_launch with the path given: AUTO takes the split path when the
// library chooses it and the workspace holds it, else the fused kernel; FUSED
// always takes the fused kernel; SPLIT takes the split path or returns
// KDA_ERR_WORKSPACE (never falls back).
static int chunk_launch_path(const KdaArgs *args, void *workspace, size_t workspace_bytes, cudaStream_t st,
                             int path) {
    bool empty = false;
    const int chk = chunk_check(args, &empty);
    if (chk != KDA_OK || empty) return chk;
    int rc;
    const bool ws_split = workspace != nullptr && (reinterpret_cast<uintptr_t>(workspace) & 255u) == 0 &&
                          workspace_bytes >=
                              split_layout(args->num_req, args->num_tokens, args->head_count, args->head_dim).total;
    bool split = false;
    if (path == KDA_CHUNK_SPLIT) {
        if (!split_ok(args->num_req) || !ws_split) return KDA_ERR_WORKSPACE;
        split = true;
    } else if (path == KDA_CHUNK_AUTO) {
        split = want_split(args->num_req, args->head_count, args->num_tokens) && ws_split;
    }
    if (split) {
        uint8_t *ws = static_cast<uint8_t *>(workspace);
        if (args->head_dim == 128)
            rc = args->gate_mode == KDA_GATE_RAW ? launch_chunk_split<128, KDA_GATE_RAW>(args, ws, st)
                                                 : launch_chunk_split<128, KDA_GATE_LOG>(args, ws, st);
        else
            rc = args->gate_mode == KDA_GATE_RAW ? launch_chunk_split<64, KDA_GATE_RAW>(args, ws, st)
                                                 : launch_chunk_split<64, KDA_GATE_LOG>(args, ws, st);
        if (rc != KDA_OK) return rc;
        return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
    }
    // The fused kernel needs only the longest-first request order (batches
    // of more than 1024 requests run in batch order, with no workspace).
    const size_t need = args->num_req <= 1024 ? order_bytes(args->num_req) : 0;
    int32_t *order = nullptr;
    if (need > 0) {
        if (workspace == nullptr || workspace_bytes < need) return KDA_ERR_WORKSPACE;
        if ((reinterpret_cast<uintptr_t>(workspace) & 3u) != 0) return KDA_ERR_ALIGNMENT;
        order = static_cast<int32_t *>(workspace);
    }
    // The library's own choice hands requests of 1..kShortLen tokens (decode
    // and verify requests in a mixed batch) to the token recurrence, where a
    // token costs one step instead of a whole 64-row chunk; the chunk kernel
    // skips them. A forced fused path runs every request through the chunk
    // kernel.
    int32_t skip_hi = 0;
    if (path == KDA_CHUNK_AUTO) {
        // The recurrence wants 16-byte aligned dt_bias for the raw gate, which
        // the chunk kernel does not: without it every request stays here.
        rc = recurrent_launch_range(args, 1, kShortLen, st);
        if (rc == KDA_OK)
            skip_hi = kShortLen;
        else if (rc != KDA_ERR_ALIGNMENT)
            return rc;
    }
    if (args->head_dim == 128)
        rc = args->gate_mode == KDA_GATE_RAW ? launch_chunk<128, KDA_GATE_RAW>(args, order, st, skip_hi)
                                             : launch_chunk<128, KDA_GATE_LOG>(args, order, st, skip_hi);
    else
        rc = args->gate_mode == KDA_GATE_RAW ? launch_chunk<64, KDA_GATE_RAW>(args, order, st, skip_hi)
                                             : launch_chunk<64, KDA_GATE_LOG>(args, order, st, skip_hi);
    if (rc != KDA_OK) return rc;
    return cudaGetLastError() == cudaSuccess ? KDA_OK : KDA_ERR_LAUNCH;
}
}  // namespace kda

extern "C" int kda_chunk_launch(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream) {
    return kda::chunk_launch_path(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), KDA_CHUNK_AUTO);
}

extern "C" int kda_chunk_launch_path(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream,
                                     int32_t path) {
    if (path != KDA_CHUNK_AUTO && path != KDA_CHUNK_FUSED && path != KDA_CHUNK_SPLIT) return KDA_ERR_INVALID_ARGUMENT;
    return kda::chunk_launch_path(args, workspace, workspace_bytes, static_cast<cudaStream_t>(stream), path);
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
    // array needs no clearing; only concurrent calls would interfere. The
    // array holds the request order alone, so this entry point always runs
    // the fused kernel (the split path's records need a caller workspace).
    return kda::chunk_launch_path(args, scratch, sizeof(int32_t) * KDA_CHUNK_STATIC_MAX_REQUESTS,
                                  static_cast<cudaStream_t>(stream), KDA_CHUNK_FUSED);
}
