/*
 * kda_b200.h -- C ABI of the B200 (sm_100a) GLM KDA varlen operator.
 *
 * Plain pointers, sizes and strides; no torch types. Every entry point is
 * asynchronous on the given CUDA stream (a cudaStream_t passed as void*),
 * never synchronises the host, never allocates, and returns a KdaStatus.
 * Device-side failures (a bounded wait that gave up) are reported through the
 * optional `status` word, which the caller reads after the stream drains.
 *
 * The entry points replace the reference's host-to-kernel seam:
 *   KdaArgs                         <- KdaLaunchArgs
 *       (sgl-glm53-ascend-ops/csrc/kda/recurrent/kda_varlen_recurrent.h:59-92)
 *       and KdaChunkLaunchArgs
 *       (sgl-glm53-ascend-ops/csrc/kda/chunk/kda_varlen_chunk.h:120-141)
 *   kda_recurrent_launch            <- LaunchKdaDecodeH16/H32/H64 and
 *       LaunchKdaPrefillH4/H8 (kda_varlen_recurrent.h:94-98), selected at
 *       kda_varlen_recurrent.cpp:218-253
 *   kda_chunk_workspace_bytes       <- the per-block workspace sizing
 *       kda_chunk::kWorkspaceFloatsPerBlock (kda_varlen_chunk.h:79-116) and
 *       its allocation at kda_varlen_chunk.cpp:154-166
 *   kda_chunk_launch                <- LaunchKdaVarlenChunk
 *       (kda_varlen_chunk.h:143-144; launched at kda_varlen_chunk.cpp:190-191)
 *   kda_prepared_recurrent_launch   <- the prepared_recurrent_kernel_* launches
 *       (sgl-glm53-ascend-ops/csrc/kda/prepared_recurrent.cpp:684-710)
 *   kda_commit_intermediate_launch  <- sgl_kernel_npu move_intermediate_cache_kda,
 *       the speculative commit called at
 *       sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:93-99
 *
 * Layouts (all row-major, element strides):
 *   q, k, v, a, g, out : [T, H, D]   (the torch [1, T, H, D] contiguous tensor)
 *   b, beta            : [T, H]
 *   A_log              : [H];  dt_bias : [H * D]
 *   state pool         : element (slot, h, k, v) at
 *                        slot*s[0] + h*s[1] + k*s[2] + v*s[3]; the production
 *                        pool is K-contiguous (s[2] == 1, s[3] == D)
 *   intermediate       : element (req, step, h, k, v) at
 *                        req*m[0] + step*m[1] + h*m[2] + k*m[3] + v*m[4]
 *   indices, cu_seqlens, track_indices, track_lens : int32 or int64
 *                        (index_bytes[] = 4 or 8 each)
 * Slot 0 of the pool is the padding row: it reads as a zero state and is never
 * written.
 */
#ifndef KDA_B200_H
#define KDA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define KDA_ABI_VERSION 1

typedef enum KdaStatus {
    KDA_OK = 0,
    KDA_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size or dimension */
    KDA_ERR_UNSUPPORTED = 2,      /* head_dim other than 64/128, ... */
    KDA_ERR_ALIGNMENT = 3,        /* a pointer or stride breaks a 16-byte rule */
    KDA_ERR_WORKSPACE = 4,        /* workspace missing or smaller than required */
    KDA_ERR_LAUNCH = 5,           /* the CUDA launch itself failed */
    KDA_ERR_TOO_LARGE = 6         /* beyond a fixed in-library capacity */
} KdaStatus;

/* Codes a kernel may write into *status (first error wins). */
#define KDA_DEVICE_ERR_WAIT_TIMEOUT 0x101  /* a bounded mbarrier wait expired */
#define KDA_DEVICE_ERR_BAD_SLOT     0x102  /* a slot index outside [0, num_slots) */
#define KDA_DEVICE_ERR_BAD_SEQLENS  0x103  /* cu_seqlens not monotone / beyond T */
#define KDA_DEVICE_ERR_GATE_RANGE   0x104  /* a 16-row gate span beyond the chunk
                                              kernel's exponent range */

typedef enum KdaGateMode {
    /* g = lower_bound * sigmoid(exp(A_log[h]) * (a + dt_bias[h])), beta =
     * sigmoid(b); q, k normalised in the kernel (kda_python.py:16-39). */
    KDA_GATE_RAW = 0,
    /* g (fp32 log-decay [T,H,D]) and beta (fp32 [T,H]) given directly; q, k
     * still normalised in the kernel. */
    KDA_GATE_LOG = 1,
    /* prepared_recurrent: q, k are fp32 and already normalised/scaled, g holds
     * exp(gate) (fp32), beta fp32; nothing is recomputed. */
    KDA_GATE_PREPARED = 2
} KdaGateMode;

typedef struct KdaArgs {
    const void *q;            /* bf16, or fp32 under KDA_GATE_PREPARED */
    const void *k;            /* bf16, or fp32 under KDA_GATE_PREPARED */
    const void *v;            /* bf16 */
    const void *a;            /* bf16 [T,H,D]  (RAW) */
    const void *b;            /* bf16 [T,H]    (RAW) */
    const float *A_log;       /* [H]           (RAW) */
    const float *dt_bias;     /* [H*D]         (RAW) */
    const float *g;           /* [T,H,D] log-decay (LOG) or exp(g) (PREPARED) */
    const float *beta;        /* [T,H]         (LOG, PREPARED) */
    void *out;                /* bf16 [T,H,D], written for every token */
    float *state;             /* fp32 pool, updated in place */
    int64_t state_stride[4];  /* slot, head, k, v */
    int64_t num_slots;        /* pool rows; slots are checked against it */
    const void *indices;      /* [num_req] pool slot per request */
    const void *cu_seqlens;   /* [num_req + 1] packed sequence boundaries */
    const void *track_indices;/* [num_req] or NULL: prefix-checkpoint slot */
    const void *track_lens;   /* [num_req] or NULL: tokens before the checkpoint */
    float *intermediate;      /* recurrent only: per-step checkpoints or NULL */
    int64_t mid_stride[5];    /* req, step, head, k, v */
    int32_t index_bytes[4];   /* indices, cu_seqlens, track_indices, track_lens */
    int32_t num_req;
    int32_t num_tokens;       /* T */
    int32_t num_heads;        /* H of the token tensors and the pool */
    int32_t head_dim;         /* D = K = V: 64 or 128 */
    int32_t head_begin;       /* heads processed: [head_begin, head_begin+head_count) */
    int32_t head_count;
    int32_t gate_mode;        /* KdaGateMode */
    float scale;              /* applied to q after the L2 norm */
    float lower_bound;        /* RAW gate bound (negative) */
    int32_t *status;          /* optional device word for KDA_DEVICE_ERR_* */
    int32_t out_fp32;         /* verification: nonzero -> `out` is fp32 [T,H,D],
                                 the pre-cast values of the bf16 output */
} KdaArgs;

/* ABI version compiled into the library (KDA_ABI_VERSION). */
int kda_abi_version(void);

/* Human-readable name of a KdaStatus or KDA_DEVICE_ERR_* code. */
const char *kda_status_string(int code);

/* Token-at-a-time recurrence: decode (one or more tokens per request, the
 * EAGLE verify regime with `intermediate`) and recurrent prefill. Persistent
 * CTAs walk (request, head, 32-row value slice) items through a ring of
 * shared-memory stages filled by bulk TMA copies. Every token row of `out`
 * for the heads processed is written: tokens no request covers, and the
 * tokens of a request rejected by the slot bounds check, as zeros.
 * Replaces LaunchKdaDecodeH{16,32,64} and LaunchKdaPrefillH{4,8}
 * (kda_varlen_recurrent.h:94-98). */
int kda_recurrent_launch(const KdaArgs *args, void *stream);

/* Bytes of device workspace kda_chunk_launch needs for these sizes (replaces
 * kda_chunk::kWorkspaceFloatsPerBlock, kda_varlen_chunk.h:79-116).
 * `num_heads` is the number of heads ONE launch processes, i.e. the
 * `head_count` the launch's KdaArgs will carry (not the H of the tensors).
 * For batches of few long sequences (requests x heads at most half the SM
 * count, >= 8 chunks per request on average) this is the size of the split
 * path's per-chunk records and state splits, ~210 KB per chunk and head at
 * D = 128 (plus a few MB of segment-boundary states); otherwise a few bytes
 * per request. The split-path size depends on the SM count of the current
 * device, so query it on the device that launches. */
size_t kda_chunk_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads, int32_t head_dim);

/* Chunk-64 WY/UT prefill over a varlen batch, any sequence lengths. The
 * workspace must be at least kda_chunk_workspace_bytes(...) bytes; its
 * contents need no initialisation. Replaces LaunchKdaVarlenChunk
 * (kda_varlen_chunk.h:143-144). `intermediate` must be NULL.
 * Two internal paths give the same results within the fp32 tolerances: a
 * fused kernel (one CTA per (sequence, head) through every chunk) and, for
 * few long sequences, a split path: a prep kernel over all (chunk, head)
 * pairs, a state scan that cuts long sequences into segments scanned side by
 * side and then chained, and an output kernel over all (chunk, head) pairs.
 * The choice depends only on the call's sizes and the device's SM count; the
 * split path runs only when the workspace holds it (256-byte aligned), else
 * the fused kernel. On the fused path, requests of 1..16 tokens (decode or
 * verify requests in a mixed batch) are computed in the same call by the
 * token recurrence of kda_recurrent_launch, launched first on the stream. */
int kda_chunk_launch(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream);

/* Which internal path a chunk launch takes (kda_chunk_launch_path). */
typedef enum KdaChunkPath {
    KDA_CHUNK_AUTO = 0,   /* the library's choice, as kda_chunk_launch */
    KDA_CHUNK_FUSED = 1,  /* always the fused kernel */
    KDA_CHUNK_SPLIT = 2   /* always the split path (at most 1024 requests) */
} KdaChunkPath;

/* Verification hook, no counterpart in the reference: kda_chunk_launch with
 * the path forced, so tests can run every case on both paths. A forced split
 * whose workspace is smaller than kda_chunk_path_workspace_bytes(...,
 * KDA_CHUNK_SPLIT) returns KDA_ERR_WORKSPACE instead of falling back. */
int kda_chunk_launch_path(const KdaArgs *args, void *workspace, size_t workspace_bytes, void *stream,
                          int32_t path);

/* Workspace bytes kda_chunk_launch_path needs for `path` (0 for an unknown
 * path); for KDA_CHUNK_AUTO the same as kda_chunk_workspace_bytes. */
size_t kda_chunk_path_workspace_bytes(int32_t num_req, int32_t num_tokens, int32_t num_heads, int32_t head_dim,
                                      int32_t path);

/* Measurement hook, no counterpart in the reference: the split path of
 * kda_chunk_launch with six caller-created cudaEvent_t handles recorded on
 * the stream -- before the plan, then after the prep kernel, the scan's
 * first pass, the combine of the segment transfers, the rescan and the
 * output kernel -- so a benchmark can report the inter-chunk state pass on
 * its own. Same arguments and results as kda_chunk_launch otherwise;
 * KDA_ERR_UNSUPPORTED when the batch would take the fused kernel,
 * KDA_ERR_WORKSPACE when the workspace cannot hold the split path. */
int kda_chunk_launch_phases(const KdaArgs *args, void *workspace, size_t workspace_bytes,
                            void *stream, void *const *events, int num_events);

/* Largest batch kda_chunk_launch_no_alloc accepts (its scratch capacity). */
#define KDA_CHUNK_STATIC_MAX_REQUESTS 1024

/* kda_chunk_launch for callers that cannot provide device memory: the same
 * prefill, with its only scratch (the longest-first request order, one int32
 * per request) kept in an array compiled into the library, so this entry
 * point never allocates. It always runs the fused kernel: the split path
 * that kda_chunk_launch picks for few long sequences keeps per-chunk records
 * in the caller's workspace, which this entry point does not have. Results
 * agree with kda_chunk_launch within the fp32 tolerances on every batch, but
 * a batch of few long sequences (e.g. one 128K-token context over 4 heads)
 * runs several times slower here than through kda_chunk_launch with a full
 * workspace. It serves callers whose device memory is already
 * fully claimed by their own pools, or hosts reaching the library through an
 * FFI with no device allocator. No counterpart in the reference, which always
 * allocates its workspace per call.
 *   - num_req above KDA_CHUNK_STATIC_MAX_REQUESTS returns KDA_ERR_TOO_LARGE.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress) with that device current; make that first call
 *     before any stream capture.
 *   - All calls on a device share the one array and it keeps the last call's
 *     contents (each call rewrites what it reads); calls that overlap on the
 *     GPU, e.g. on two streams, race on it and must be serialised. */
int kda_chunk_launch_no_alloc(const KdaArgs *args, void *stream);

/* The recurrence on prepared fp32 inputs (gate_mode is forced to
 * KDA_GATE_PREPARED). Replaces the prepared_recurrent_kernel_* launches
 * (prepared_recurrent.cpp:578-604, 684-710). */
int kda_prepared_recurrent_launch(const KdaArgs *args, void *stream);

/* Speculative-decoding commit. A verify pass (kda_recurrent_launch with
 * `intermediate`) leaves one checkpoint per draft step; once the number of
 * accepted tokens is known, entry i copies, for every layer l and head h,
 *     dst[l, dst_indices[i], h] <- src[l, src_indices[i], step_indices[i], h]
 * (each a D x D fp32 block, element (r, c) at r*s[...-2] + c*s[...-1]).
 * Replaces sgl_kernel_npu's move_intermediate_cache_kda, the commit the
 * reference's MTP test runs after a verify
 * (sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:87-99).
 *   - An entry whose step index is negative (no token accepted) copies nothing.
 *   - A slot, request or step index past its dimension copies nothing and
 *     writes KDA_DEVICE_ERR_BAD_SLOT into *status (when status is non-NULL).
 *   - Entries must name distinct destinations; the copy order among entries
 *     is unspecified. */
typedef struct KdaCommitArgs {
    float *dst;                   /* pool: [layers][slots][H][D][D] by dst_stride */
    const float *src;             /* checkpoints: [layers][requests][steps][H][D][D] */
    int64_t dst_stride[5];        /* layer, slot, head, row, column (elements) */
    int64_t src_stride[6];        /* layer, request, step, head, row, column */
    const void *dst_indices;      /* [num_entries] pool slot */
    const void *src_indices;      /* [num_entries] request row of src */
    const void *step_indices;     /* [num_entries] accepted draft step, or < 0 */
    int32_t index_bytes[3];       /* 4 or 8 each */
    int32_t num_entries;
    int32_t num_layers;
    int32_t num_heads;
    int32_t head_dim;             /* D, any value >= 1 */
    int64_t num_slots;            /* dst slots */
    int32_t num_requests;         /* src requests */
    int32_t num_steps;            /* src steps */
    int32_t *status;              /* optional device word for KDA_DEVICE_ERR_* */
} KdaCommitArgs;

int kda_commit_intermediate_launch(const KdaCommitArgs *args, void *stream);

/* Self-test of the bounded waits, no counterpart in the reference (whose
 * kernels wait without a limit). One CTA of 64 threads makes `waits` (1..64)
 * successive waits, of at most `polls` polls each (a poll suspends for up to
 * ~1 us), on an mbarrier that nothing arrives on: the same bounded wait every
 * kernel of this library uses. With `give_up` nonzero the CTA-wide give-up
 * word is used, as the chunk kernels use it: after the first expiry the
 * remaining waits give up at their first poll. Each expired wait writes
 * KDA_DEVICE_ERR_WAIT_TIMEOUT into *status (first error wins) and adds one to
 * *expired (both device int32); the kernel then ends normally and the context
 * stays usable. */
int kda_selftest_wait_timeout(int32_t *status, int32_t *expired, int32_t polls, int32_t waits, int32_t give_up,
                              void *stream);

/* ---- Causal-conv front end ---------------------------------------------
 * The short depthwise causal convolution the attention layer runs over the
 * mixed q | k | v projection before the KDA op, with its conv-state pool.
 * Replaces the causal_conv1d step of sglang's attention backend
 * (AscendKDAAttnBackend.forward_extend, run by
 * sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387;
 * the conv code itself is sglang's and not in the reference tree):
 *   out[t, c] = act(bias[c] + sum_{k<W} weight[c, k] * xin[t + k, c]),
 * xin = the W-1 rows before the request's first token, then its tokens.
 * Rules:
 *   - The conv state of a slot is `window` (W-1 <= window <= 8) raw input
 *     rows, oldest first. A request that continues (has_initial nonzero, or
 *     has_initial NULL) reads the last W-1 rows of its slot as the rows before
 *     its first token; one that does not reads zeros. After the call the slot
 *     holds the last `window` rows of (old window, or zeros, ++ the request's
 *     tokens); an empty request leaves it unchanged.
 *   - Tracked-prefix checkpoint: with track_indices[r] > 0 and
 *     0 <= track_lens[r] <= the request's length, that slot receives the
 *     `window` rows ending after the first track_lens[r] tokens (rows before
 *     the request from the old window, or zeros). A tracked length outside
 *     that range takes no checkpoint.
 *   - Slot 0 is the padding row: it reads as zeros and is never written.
 *   - A slot or checkpoint slot outside [0, num_slots), or a malformed
 *     cu_seqlens entry, rejects the request: KDA_DEVICE_ERR_BAD_SLOT /
 *     _BAD_SEQLENS in *status, zero output rows, no state written.
 *   - Every token row of `out` is written: zeros where no request covers it.
 *   - The requests' slots and checkpoint slots must all be distinct.
 * Layouts: x bf16 [T][x_row_stride] (channels contiguous); weight fp32
 * [channels][width]; bias fp32 [channels] or NULL; conv state bf16, element
 * (slot, row, channel) at slot*s[0] + row*s[1] + channel; out bf16
 * [num_parts][T][channels / num_parts] (num_parts = 3: contiguous q, k, v
 * planes, the [T, H, D] tensors the KDA op reads). channels / num_parts, the
 * row strides and both pool strides must be multiples of 8 elements, and the
 * x, out, state, weight and bias pointers 16-byte aligned (else
 * KDA_ERR_ALIGNMENT). */
#define KDA_CONV_ACT_NONE 0
#define KDA_CONV_ACT_SILU 1

typedef struct KdaConvArgs {
    const void *x;              /* bf16 [T][x_row_stride]: the mixed projection */
    int64_t x_row_stride;       /* elements, >= channels */
    const float *weight;        /* fp32 [channels][width] */
    const float *bias;          /* fp32 [channels] or NULL */
    void *conv_state;           /* bf16 pool, updated in place */
    int64_t state_stride[2];    /* slot, row (elements) */
    int64_t num_slots;
    int32_t window;             /* rows per slot, width - 1 .. 8 */
    const void *indices;        /* [num_req] slot per request */
    const void *cu_seqlens;     /* [num_req + 1] packed sequence boundaries */
    const void *has_initial;    /* [num_req] nonzero: continue from the slot; NULL: all continue */
    const void *track_indices;  /* [num_req] or NULL: checkpoint slot (0: none) */
    const void *track_lens;     /* [num_req] or NULL: tokens before the checkpoint */
    int32_t index_bytes[5];     /* indices, cu_seqlens (4|8), has_initial (1|4|8), track_indices, track_lens (4|8) */
    int32_t num_req;
    int32_t num_tokens;         /* T */
    int32_t channels;           /* C */
    int32_t width;              /* W: 1..4 taps */
    int32_t num_parts;          /* output planes */
    int32_t activation;         /* KDA_CONV_ACT_NONE or KDA_CONV_ACT_SILU */
    void *out;                  /* bf16 [num_parts][T][channels / num_parts] */
    int32_t *status;            /* optional device word for KDA_DEVICE_ERR_* */
} KdaConvArgs;

/* The conv front end over a varlen batch (prefill, decode and verify requests
 * alike): two kernels on the stream, one per request (state work and each
 * request's first W-1 outputs) and one per 64 tokens (the other outputs).
 * With no requests it zeroes `out`. */
int kda_conv_launch(const KdaConvArgs *args, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* KDA_B200_H */
