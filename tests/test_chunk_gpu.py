"""GPU parity of the chunk-64 prefill kernel against the CPU oracle.

Ports the reference's tests/ops/test_kda_chunk.py (its ten CASES: one/several
chunks and sequences, the zero slot, tracked checkpoints before, inside, on the
boundary of and at the end of a chunk; untouched slots) and adds what the B200
op supports beyond it: lengths that are not multiples of 64, any head count,
K = V = 64, the log-gate entry point, BASELINE config 3 at full size, int64
metadata and CUDA-graph replay. Every oracle test runs twice: through the
torch op with the library's own choice between the fused kernel and the split
path (prep + scan kernels), and through the C ABI with the split path forced
(kda_chunk_launch_path), so both are covered. BASELINE configs 3 and 4 are
checked on every head against the oracle, and configs 3, 5 and a tracked case
also through the kernel's fp32 pre-cast output, at the output bar with no
rounding credit. Tolerances: tests/kda_checks.py.
"""

import pytest
import torch

from chunk_abi import chunk_via_abi
from golden_io import bf16, expected_pool, kcontig, load, raw_kwargs
from kda_checks import assert_out_close, assert_state_close, assert_untouched, clone_pool
from oracle import kda_ref

KDA_CHUNK_AUTO, KDA_CHUNK_FUSED, KDA_CHUNK_SPLIT = 0, 1, 2   # KdaChunkPath

pytestmark = pytest.mark.gpu
DEV = "cuda"
SLOTS = 8


@pytest.fixture(scope="module")
def ops():
    from sgl_glm53_ascend_ops import ops as _ops
    return _ops


@pytest.fixture(params=["auto", "split"])
def chunk_path(request):
    """"auto": the torch op, with the library's own path choice; "split": the
    C ABI with the split path forced."""
    return request.param


def _run(ops, dkw, path):
    """One chunk prefill on device kwargs: the torch op (raw or log gate) for
    "auto", kda_chunk_launch_path with the split path forced for "split"."""
    if path == "split":
        return chunk_via_abi(dkw, KDA_CHUNK_SPLIT)
    op = ops.kda_varlen_chunk if "a" in dkw else ops.kda_varlen_chunk_g
    out = op(**dkw, prefill=True)
    torch.cuda.synchronize()
    return out


def _dev(kw):
    out = {}
    for n, t in kw.items():
        if isinstance(t, torch.Tensor):
            out[n] = t.transpose(-1, -2).to(DEV).transpose(-1, -2) if n == "initial_state_source" else t.to(DEV)
        else:
            out[n] = t
    return out


def _case(heads, cu_seqlens, slots, track=None, seed=0, D=128, lower_bound=-5.0):
    """test_kda_chunk.py:59-88 inputs (0.2-scaled bf16, nonzero K-contiguous pool)."""
    torch.manual_seed(20261103 + seed)
    tokens = cu_seqlens[-1]
    kw = {n: (torch.randn(1, tokens, heads, D) * 0.2).bfloat16() for n in ("q", "k", "v", "a")}
    kw["b"] = torch.randn(1, tokens, heads).bfloat16()
    kw["A_log"] = torch.randn(heads) * 0.1
    kw["dt_bias"] = torch.randn(heads, D) * 0.1
    kw["initial_state_source"] = (torch.randn(SLOTS, heads, D, D) * 0.1).transpose(-1, -2)
    kw["initial_state_indices"] = torch.tensor(slots, dtype=torch.int32)
    kw["cu_seqlens"] = torch.tensor(cu_seqlens, dtype=torch.int32)
    kw["lower_bound"] = lower_bound
    kw["scale"] = D ** -0.5
    if track is not None:
        kw["track_state_indices"] = torch.tensor(track[0], dtype=torch.int32)
        kw["track_state_lens"] = torch.tensor(track[1], dtype=torch.int32)
    return kw


def _check(ops, kw, touched, path):
    dkw = _dev(kw)
    out = _run(ops, dkw, path)
    ref_pool = clone_pool(kw["initial_state_source"])
    ref = kda_ref.kda_varlen_chunk(**dict(kw, initial_state_source=ref_pool), out_fp32=True)
    got = dkw["initial_state_source"].cpu()
    assert_out_close(out.cpu(), ref)
    for s in touched:
        assert_state_close(got[s], ref_pool[s], what=f"slot {s}")
    assert_untouched(got, kw["initial_state_source"], touched)


# (label, heads, cu_seqlens, slots, track) -- test_kda_chunk.py:203-214
CASES = [
    ("one chunk", 1, [0, 64], [1], None),
    ("two chunks", 1, [0, 128], [1], None),
    ("four chunks", 2, [0, 256], [1], None),
    ("two sequences", 2, [0, 128, 256], [1, 2], None),
    ("ragged varlen", 1, [0, 64, 192, 256], [1, 2, 3], None),
    ("zero slot", 1, [0, 128], [0], None),
    ("track at 0", 2, [0, 128], [1], ([4], [0])),
    ("track mid-chunk", 2, [0, 128], [1], ([4], [32])),
    ("track on boundary", 2, [0, 128], [1], ([4], [64])),
    ("track at end", 1, [0, 192], [1], ([4], [192])),
]


@pytest.mark.parametrize("label,heads,cu_seqlens,slots,track", CASES, ids=[c[0].replace(" ", "-") for c in CASES])
def test_chunk_matches_oracle(ops, chunk_path, label, heads, cu_seqlens, slots, track):
    kw = _case(heads, cu_seqlens, slots, track, seed=len(label))
    touched = {s for s in slots if s > 0} | ({track[0][0]} if track else set())
    _check(ops, kw, touched, chunk_path)


def test_chunk_leaves_other_slots_untouched(ops, chunk_path):
    kw = _case(2, [0, 128], [3])
    _check(ops, kw, {3}, chunk_path)


# Lengths the reference rejects (kda_varlen_chunk.cpp:139-142): any length.
RAGGED = [
    ([0, 1], [1], None),
    ([0, 37], [2], None),
    ([0, 100], [1], ([3], [77])),
    ([0, 63, 65, 65, 200], [1, 2, 5, 3], ([4, 0, 6, 7], [63, 0, 0, 135])),
    ([0, 129, 130, 387], [0, 2, 1], ([5, 6, 0], [129, 1, 0])),
]


@pytest.mark.parametrize("cu_seqlens,slots,track", RAGGED, ids=lambda x: str(x))
@pytest.mark.parametrize("D", (64, 128))
def test_ragged_lengths_match_oracle(ops, chunk_path, cu_seqlens, slots, track, D):
    kw = _case(3, cu_seqlens, slots, track, seed=sum(cu_seqlens), D=D)
    touched = {s for s in slots if s > 0} | ({s for s in track[0] if s > 0} if track else set())
    _check(ops, kw, touched, chunk_path)


# The op's own choice hands requests of 1..16 tokens to the token recurrence
# and the rest to the chunk kernel, in one call: lengths on both sides of the
# boundary, an empty request, the padding slot and prefix checkpoints in short
# requests (at 0, inside, at the end) and in a long one.
ROUTED = [
    ([0, 1, 17, 33, 49, 129], [1, 2, 3, 4, 5], None),
    ([0, 16, 16, 31, 32, 200], [1, 0, 2, 3, 4], ([6, 0, 7, 0, 5], [0, 0, 15, 0, 100])),
    ([0, 3, 7, 23, 87, 91], [2, 1, 3, 4, 5], ([6, 7, 0, 0, 0], [3, 2, 0, 0, 0])),
]


@pytest.mark.parametrize("cu_seqlens,slots,track", ROUTED, ids=lambda x: str(x))
@pytest.mark.parametrize("D", (64, 128))
def test_short_requests_routed_to_recurrence(ops, cu_seqlens, slots, track, D):
    kw = _case(4, cu_seqlens, slots, track, seed=sum(cu_seqlens) + D, D=D)
    touched = {s for s in slots if s > 0} | ({s for s in track[0] if s > 0} if track else set())
    _check(ops, kw, touched, "auto")
    # the forced fused kernel (every request through the chunk kernel) agrees
    a, b = _dev(kw), _dev(kw)
    oa = _run(ops, a, "auto")
    ob = chunk_via_abi(b, KDA_CHUNK_FUSED)
    assert_out_close(oa.cpu(), ob.cpu())
    assert_state_close(a["initial_state_source"].cpu(), b["initial_state_source"].cpu())


@pytest.mark.parametrize("name", ["chunk_raw_tracked", "chunktest_ragged_varlen", "chunktest_zero_slot",
                                  "chunktest_track_at_0", "chunktest_track_mid_chunk", "chunktest_track_at_end"])
def test_chunk_matches_reference_golden(ops, chunk_path, name):
    f = load(name)
    kw = raw_kwargs(f)
    kw["initial_state_source"] = kcontig(f["pool_in"])
    dkw = _dev(kw)
    out = _run(ops, dkw, chunk_path)
    ref_out = torch.from_numpy(f["out"])
    if name == "chunk_raw_tracked":
        ref_out = ref_out.bfloat16()              # kda_chunk_torch returned bf16
    assert_out_close(out.cpu(), ref_out)
    pool = dkw["initial_state_source"].cpu()
    assert_state_close(pool, expected_pool(f))
    assert_untouched(pool, torch.from_numpy(f["pool_in"]), f["pool_out_slots"])


@pytest.mark.parametrize("lower_bound", (-1.0, -5.0, -10.0))
def test_gate_strength(ops, chunk_path, lower_bound):
    """Gates down to -10 per step: the 16-row anchors keep every factor in range."""
    kw = _case(2, [0, 200, 328], [1, 2], seed=3, lower_bound=lower_bound)
    _check(ops, kw, {1, 2}, chunk_path)


def test_loggate_matches_oracle(ops, chunk_path):
    import kda_workloads as workloads
    w = workloads.config3(heads=4, lengths=[700, 64, 1, 333])
    w.pool = (torch.randn(w.pool.shape[0], 4, 128, 128) * 0.1).transpose(-1, -2)
    d = w.to(DEV)
    out = _run(ops, d.kwargs(), chunk_path)
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_chunk_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out.cpu(), ref)
    assert_state_close(d.pool.cpu()[1:], ref_pool[1:])


# Requests long enough (and heads few enough) that the split path cuts them
# into segments: a first pass from zero and from the identity per segment
# (leaving midpoint states too), the combine of the segment transfers, and a
# rescan of each segment as two halves from the true start and midpoint
# states. Mixed with short requests that stay whole; checkpoints at 0, inside
# segment 0, on a segment boundary, inside a middle and the last segment, in
# either half, at the end.
SEGMENTED = [
    (2, [0, 3000], [1], None),
    (1, [0, 3000, 3001, 5500, 6100, 8100], [1, 0, 2, 3, 7], ([4, 0, 5, 6, 0], [1024, 0, 2300, 300, 0])),
    (2, [0, 1500, 2800], [1, 2], ([3, 4], [0, 1300])),
    (3, [0, 1111, 1175], [2, 1], ([5, 6], [100, 64])),
    # 17 chunks (checkpoint in the second half of the last segment) and 65
    # chunks (a one-chunk last segment: its second half is empty, the final
    # state comes from the midpoint product alone)
    (1, [0, 1034, 5134], [1, 2], ([3, 4], [1034, 4100])),
]


@pytest.mark.parametrize("heads,cu_seqlens,slots,track", SEGMENTED, ids=lambda x: str(x))
@pytest.mark.parametrize("D", (64, 128))
def test_segmented_scan_matches_oracle(ops, chunk_path, heads, cu_seqlens, slots, track, D):
    kw = _case(heads, cu_seqlens, slots, track, seed=len(cu_seqlens) + D, D=D)
    touched = {s for s in slots if s > 0} | ({s for s in track[0] if s > 0} if track else set())
    _check(ops, kw, touched, chunk_path)


@pytest.fixture(scope="module")
def cfg3_oracle():
    """BASELINE config 3 (8 sequences, 33,494 tokens, none a multiple of 64,
    H=32) and the oracle's fp32 output and final states for all 32 heads (the
    token recurrence, exact and fast enough on the CPU)."""
    import kda_workloads as workloads
    w = workloads.config3()
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    return w, ref, ref_pool


@pytest.mark.parametrize("path", ["auto", "split"])
def test_cfg3_full_size(ops, cfg3_oracle, path):
    """Config 3 at full size, every head: output and the 8 final states against
    the oracle; a second run from the same pool is bit-identical."""
    w, ref, ref_pool = cfg3_oracle
    d = w.to(DEV)
    pool0 = clone_pool(d.pool)
    out = _run(ops, d.kwargs(), path)
    pool_a = clone_pool(d.pool)
    d.pool.copy_(pool0)
    out_b = _run(ops, d.kwargs(), path)
    assert torch.equal(out, out_b) and torch.equal(pool_a, d.pool), "not deterministic"
    got = out.cpu()
    for h0 in range(0, 32, 4):
        assert_out_close(got[:, :, h0:h0 + 4], ref[:, :, h0:h0 + 4], what=f"output heads {h0}..{h0 + 3}")
    assert_state_close(pool_a[1:].cpu(), ref_pool[1:])


@pytest.mark.parametrize("path", [KDA_CHUNK_FUSED, KDA_CHUNK_SPLIT], ids=["fused", "split"])
def test_cfg3_fp32_output(ops, cfg3_oracle, path):
    """Config 3, every head, through the kernel's fp32 pre-cast output: max-abs
    error <= 5e-3 of the output RMS with no rounding credit."""
    w, ref, ref_pool = cfg3_oracle
    d = w.to(DEV)
    out = chunk_via_abi(d.kwargs(), path, out_fp32=True)
    assert out.dtype == torch.float32
    assert_out_close(out.cpu(), ref, what="fp32 output")
    assert_state_close(d.pool.cpu()[1:], ref_pool[1:])


def test_chunk_equals_recurrent_kernel(ops):
    """The two GPU paths agree on the same inputs (prefill through both)."""
    kw = _case(4, [0, 150, 300], [1, 2], seed=9)
    a = _dev(kw)
    b = _dev(kw)
    oa = ops.kda_varlen_chunk(**a, prefill=True)
    ob = ops.kda_varlen_recurrent(**b, prefill=True)
    torch.cuda.synchronize()
    assert_out_close(oa.cpu(), ob.cpu())          # both bf16: one-ulp credit
    assert_state_close(a["initial_state_source"].cpu()[1:3], b["initial_state_source"].cpu()[1:3])


def test_int64_metadata_bitwise(ops):
    kw = _case(2, [0, 70, 200], [1, 2], ([3, 0], [50, 0]), seed=2)
    a = _dev(kw)
    b = _dev(dict(kw, initial_state_indices=kw["initial_state_indices"].long(),
                  cu_seqlens=kw["cu_seqlens"].long(), track_state_indices=kw["track_state_indices"].long(),
                  track_state_lens=kw["track_state_lens"].long()))
    oa = ops.kda_varlen_chunk(**a, prefill=True)
    ob = ops.kda_varlen_chunk(**b, prefill=True)
    torch.cuda.synchronize()
    assert torch.equal(oa, ob)
    assert torch.equal(a["initial_state_source"], b["initial_state_source"])


def test_chunk_launch_phases_matches_launch(ops):
    """The measurement hook runs the same split path: bit-identical outputs and
    pool, six ordered events; a batch that takes the fused kernel is refused."""
    from sgl_glm53_ascend_ops import abi
    kw = _case(2, [0, 3000, 3001], [1, 2], ([3, 0], [1024, 0]), seed=41)
    runs = []
    for phases in (False, True):
        d = _dev(kw)
        pool = d["initial_state_source"]
        out = torch.empty(d["v"].shape, dtype=torch.bfloat16, device=DEV)
        a = abi.args_from_tensors(q=d["q"], k=d["k"], v=d["v"], out=out, state=pool,
                                  indices=d["initial_state_indices"], cu_seqlens=d["cu_seqlens"], scale=d["scale"],
                                  gate_mode=abi.KDA_GATE_RAW, a=d["a"], b=d["b"], A_log=d["A_log"],
                                  dt_bias=d["dt_bias"], lower_bound=d["lower_bound"],
                                  track_indices=d["track_state_indices"], track_lens=d["track_state_lens"])
        n = abi.chunk_workspace_bytes(2, 3001, 2, 128)
        ws = torch.empty(n, dtype=torch.uint8, device=DEV)
        if phases:
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
            for e in ev:
                e.record()
            assert abi.chunk_launch_phases(a, ws, n, ev) == abi.KDA_OK
        else:
            assert abi.chunk_launch(a, ws, n) == abi.KDA_OK
        torch.cuda.synchronize()
        runs.append((out.cpu(), pool.cpu()))
        if phases:
            assert all(ev[i].elapsed_time(ev[i + 1]) >= 0 for i in range(5))
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])
    # 64 one-chunk requests x 32 heads: the fused kernel's batch.
    big = _dev(_case(32, [64 * i for i in range(65)], [0] * 64, seed=42))
    a = abi.args_from_tensors(q=big["q"], k=big["k"], v=big["v"], out=torch.empty_like(big["v"]),
                              state=big["initial_state_source"], indices=big["initial_state_indices"],
                              cu_seqlens=big["cu_seqlens"], scale=big["scale"], gate_mode=abi.KDA_GATE_RAW,
                              a=big["a"], b=big["b"], A_log=big["A_log"], dt_bias=big["dt_bias"],
                              lower_bound=big["lower_bound"])
    ws = torch.empty(1 << 20, dtype=torch.uint8, device=DEV)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in ev:
        e.record()
    assert abi.chunk_launch_phases(a, ws, 1 << 20, ev) == abi.KDA_ERR_UNSUPPORTED


def test_chunk_cuda_graph_replay(ops):
    """Capture once; replay with new cu_seqlens/slots/values behind the pointers
    (test_glm53_kda_prefix_ascendc.py:185-293, chunk op, no host sync)."""
    kw = _case(4, [0, 129, 194, 257], [1, 2, 3], ([5, 6, 7], [64, 32, 63]), seed=4)
    d = _dev(kw)
    initial = clone_pool(d["initial_state_source"])
    for _ in range(2):
        d["initial_state_source"].copy_(initial)
        ops.kda_varlen_chunk(**d, prefill=True)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph):
            captured = ops.kda_varlen_chunk(**d, prefill=True)
    torch.cuda.synchronize()
    for replay, lens in enumerate(([129, 65, 63], [65, 129, 63], [1, 200, 56])):
        cu = [0]
        for n in lens:
            cu.append(cu[-1] + n)
        d["cu_seqlens"].copy_(torch.tensor(cu, dtype=torch.int32))
        d["initial_state_indices"].copy_(torch.tensor([(replay + r) % 4 for r in range(3)], dtype=torch.int32))
        for name in ("q", "k", "v", "a"):
            d[name].copy_((torch.randn_like(d[name].float()) * 0.2).bfloat16())
        d["initial_state_source"].copy_(initial)
        ref_pool = clone_pool(initial)
        expected = ops.kda_varlen_chunk(**dict(d, initial_state_source=ref_pool), prefill=True)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(d["initial_state_source"], ref_pool)
        assert torch.equal(captured, expected)
    del graph


def test_cfg4_long_context(ops):
    """one 131,072-token sequence (2048 chunks), here 4 heads
    with an fp32 initial state. The op takes the split path by itself; every
    head's output and final state are checked against the oracle's token
    recurrence over the whole sequence, the run is deterministic, and the
    fused kernel (forced through the C ABI) agrees with it."""
    import kda_workloads as workloads
    w = workloads.config4(seed=4, heads=4)
    d = w.to(DEV)
    pool0 = clone_pool(d.pool)
    out = ops.kda_varlen_chunk_g(**d.kwargs(), prefill=True)
    pool_split = clone_pool(d.pool)
    d.pool.copy_(pool0)
    out_b = ops.kda_varlen_chunk_g(**d.kwargs(), prefill=True)
    torch.cuda.synchronize()
    assert torch.equal(out, out_b) and torch.equal(pool_split, d.pool), "not deterministic"
    d.pool.copy_(pool0)
    out_f = chunk_via_abi(d.kwargs(), KDA_CHUNK_FUSED)
    assert_out_close(out_f.cpu(), out.cpu())          # both bf16: one-ulp credit
    assert_state_close(d.pool.cpu()[1:], pool_split.cpu()[1:])
    got = out.cpu()
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    for h in range(4):
        assert_out_close(got[:, :, h:h + 1], ref[:, :, h:h + 1], what=f"output head {h}")
        assert_state_close(pool_split[1:, h:h + 1].cpu(), ref_pool[1:, h:h + 1], what=f"state head {h}")


@pytest.fixture(scope="module")
def cfg5_oracle():
    """64 one-token requests and 4 resumed 2048-token
    prefills (68 distinct slots of a 1024-slot pool, nonzero states), H=32,
    with the oracle's fp32 output and pool."""
    import kda_workloads as workloads
    w = workloads.config5()
    before = clone_pool(w.pool)
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    return w, before, ref, ref_pool


def test_cfg5_mixed_batch(ops, cfg5_oracle):
    """Config 5 in one chunk-op call: outputs and the 68 updated slots against
    the oracle; the 955 other slots bit-equal."""
    w, before, ref, ref_pool = cfg5_oracle
    d = w.to(DEV)
    out = ops.kda_varlen_chunk_g(**d.kwargs(), prefill=True)
    torch.cuda.synchronize()
    got = d.pool.cpu()
    del d
    assert_out_close(out.cpu(), ref)
    touched = [int(s) for s in w.indices]
    assert_state_close(got[touched], ref_pool[touched])
    assert_untouched(got, before, touched)


def test_cfg5_fp32_output(ops, cfg5_oracle):
    """Config 5 through the kernel's fp32 pre-cast output (C ABI): the output
    bar with no rounding credit, the updated slots, the untouched slots."""
    w, before, ref, ref_pool = cfg5_oracle
    d = w.to(DEV)
    out = chunk_via_abi(d.kwargs(), KDA_CHUNK_AUTO, out_fp32=True)
    got = d.pool.cpu()
    del d
    assert_out_close(out.cpu(), ref, what="fp32 output")
    touched = [int(s) for s in w.indices]
    assert_state_close(got[touched], ref_pool[touched])
    assert_untouched(got, before, touched)


@pytest.mark.parametrize("path", [KDA_CHUNK_FUSED, KDA_CHUNK_SPLIT], ids=["fused", "split"])
def test_tracked_fp32_output(ops, path):
    """Tracked checkpoints (before, inside, on the boundary of and at the end
    of a chunk, and in a segmented request) through the fp32 pre-cast output."""
    kw = _case(2, [0, 63, 65, 265, 3465], [1, 2, 5, 3], ([4, 0, 6, 7], [63, 0, 135, 1700]), seed=77)
    dkw = _dev(kw)
    out = chunk_via_abi(dkw, path, out_fp32=True)
    ref_pool = clone_pool(kw["initial_state_source"])
    ref = kda_ref.kda_varlen_chunk(**dict(kw, initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out.cpu(), ref, what="fp32 output")
    got = dkw["initial_state_source"].cpu()
    touched = {1, 2, 5, 3, 4, 6, 7}
    for s in touched:
        assert_state_close(got[s], ref_pool[s], what=f"slot {s}")
    assert_untouched(got, kw["initial_state_source"], touched)
