"""GPU parity of the recurrent (decode / verify / recurrent-prefill) kernel.

Each case runs the CUDA kernel (through the torch op or directly through the C
ABI) and ``oracle/kda_ref.py`` on the same seeded inputs. Ports the contracts
of the reference's tests/ops/test_kda_decode_numerics.py (lengths crossing
step groups, H in {16, 32, 64}, checkpoints, untouched slots),
test_kda_index_dtypes.py (int32 == int64 bit-exactly) and test_kda.py
(layout rejections), with the oracle in place of the absent sglang Triton
kernel; tolerances are in tests/kda_checks.py.
"""

import itertools

import pytest
import torch

from golden_io import bf16, expected_pool, kcontig, load, raw_kwargs
from kda_checks import (assert_out_close, assert_state_close, assert_untouched, clone_pool,
                        state_error)
from oracle import kda_ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module")
def ops():
    from sgl_glm53_ascend_ops import ops as _ops
    return _ops


@pytest.fixture(scope="module")
def abi():
    from sgl_glm53_ascend_ops import abi as _abi
    return _abi


def _dev(kw):
    out = {}
    for n, t in kw.items():
        if isinstance(t, torch.Tensor):
            out[n] = t.transpose(-1, -2).to(DEV).transpose(-1, -2) if n == "initial_state_source" else t.to(DEV)
        else:
            out[n] = t
    return out


def _raw_case(heads, lengths, D=128, slots=16, seed=0, lower_bound=-5.0):
    """Reference-style raw-gate inputs (test_kda_decode_numerics.py:56-82)."""
    tokens = sum(lengths)
    torch.manual_seed(31337 + tokens * 97 + len(lengths) + seed)
    t = {n: (torch.randn(1, tokens, heads, D) * 0.2).bfloat16() for n in ("q", "k", "v", "a")}
    t["b"] = torch.randn(1, tokens, heads).bfloat16()
    t["A_log"] = torch.randn(heads) * 0.1
    t["dt_bias"] = torch.randn(heads * D) * 0.1
    t["initial_state_source"] = (torch.randn(slots, heads, D, D) * 0.1).transpose(-1, -2)
    t["initial_state_indices"] = torch.arange(1, len(lengths) + 1, dtype=torch.int32)
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + n)
    t["cu_seqlens"] = torch.tensor(cu, dtype=torch.int32)
    t["lower_bound"] = lower_bound
    t["scale"] = D ** -0.5
    return t


def _run_op(fn, kw, **extra):
    dkw = _dev(kw)
    pool = dkw["initial_state_source"]
    out = fn(**dkw, **extra)
    torch.cuda.synchronize()
    return out.cpu(), pool.cpu()


# ---------------------------------------------------------------------------
# Golden fixtures (reference outputs) through the torch ops
# ---------------------------------------------------------------------------

def test_cfg1_loggate_matches_reference_golden(ops):
    f = load("cfg1_recurrent_loggate")
    kw = dict(q=bf16(f["q"]), k=bf16(f["k"]), v=bf16(f["v"]), g=torch.from_numpy(f["g"]),
              beta=torch.from_numpy(f["beta"]), initial_state_source=kcontig(f["pool_in"]),
              initial_state_indices=torch.from_numpy(f["indices"]),
              cu_seqlens=torch.from_numpy(f["cu_seqlens"]), scale=float(f["scale"]))
    out, pool = _run_op(ops.kda_varlen_recurrent_g, kw, prefill=True)
    assert_out_close(out, torch.from_numpy(f["out"]))
    assert_state_close(pool, expected_pool(f))
    assert_untouched(pool, torch.from_numpy(f["pool_in"]), f["pool_out_slots"])


@pytest.mark.parametrize("name", ["recur_raw_tracked_d64", "recur_raw_tracked_d128", "recur_raw_varlen"])
def test_raw_gate_matches_reference_golden(ops, name):
    f = load(name)
    kw = raw_kwargs(f)
    kw["initial_state_source"] = kcontig(f["pool_in"])
    out, pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=True)
    assert_out_close(out, torch.from_numpy(f["out"]))
    assert_state_close(pool, expected_pool(f))
    assert_untouched(pool, torch.from_numpy(f["pool_in"]), f["pool_out_slots"])


def test_intermediate_matches_reference_golden(ops):
    f = load("recur_raw_intermediate")
    kw = raw_kwargs(f)
    kw["initial_state_source"] = kcontig(f["pool_in"])
    H, D = kw["q"].shape[2], kw["q"].shape[3]
    noise = (torch.randn(3, 4, H, D, D) * 0.1).transpose(-1, -2)
    mid = noise.transpose(-1, -2).to(DEV).transpose(-1, -2)
    dkw = _dev(kw)
    out = ops.kda_varlen_recurrent(**dkw, intermediate_state=mid, prefill=False)
    torch.cuda.synchronize()
    assert_out_close(out.cpu(), torch.from_numpy(f["out"]))
    rows = f["mid_out_rows"].tolist()
    assert_state_close(mid.cpu()[rows], torch.from_numpy(f["mid_out"]), what="checkpoints")
    assert torch.equal(mid.cpu()[1], noise[1]), "slot-0 request wrote checkpoints"
    assert torch.equal(dkw["initial_state_source"].cpu(), kcontig(f["pool_in"])), "verify wrote the pool"


def test_prepared_matches_triton_golden(ops):
    f = load("prepared_triton")
    state = torch.from_numpy(f["state_in"]).to(DEV)          # [K,V]-contiguous, as v1 takes it
    out = torch.zeros(bf16(f["out"]).shape, dtype=torch.bfloat16, device=DEV)
    ops.prepared_recurrent(
        torch.from_numpy(f["qn"]).to(DEV), torch.from_numpy(f["kn"]).to(DEV), bf16(f["v"]).to(DEV),
        torch.from_numpy(f["gdecay"]).to(DEV), torch.from_numpy(f["beta"]).to(DEV), out, state,
        torch.from_numpy(f["indices"]).int().to(DEV), torch.from_numpy(f["starts"]).int().to(DEV),
        torch.from_numpy(f["track_indices"]).int().to(DEV),
        torch.from_numpy(f["track_lens"]).int().to(DEV), True, 0)
    torch.cuda.synchronize()
    assert_out_close(out.cpu(), bf16(f["out"]))
    assert_state_close(state.cpu(), torch.from_numpy(f["state_out"]))


# ---------------------------------------------------------------------------
# Decode numerics vs the oracle (test_kda_decode_numerics.py:42-53)
# ---------------------------------------------------------------------------

DECODE_CASES = [(1,), (4,), (5,), (8,), (9,), (16,), (1,) * 8, (4,) * 4, (1, 2, 3, 4, 5, 6, 7), (7, 1, 4, 9)]


@pytest.mark.parametrize("heads", (16, 32, 64))
@pytest.mark.parametrize("lengths", DECODE_CASES, ids=lambda l: "x".join(map(str, l)))
def test_decode_matches_oracle(ops, heads, lengths):
    kw = _raw_case(heads, lengths)
    before = clone_pool(kw["initial_state_source"])
    out, pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=False)
    ref_pool = clone_pool(kw["initial_state_source"])
    ref = kda_ref.kda_varlen_recurrent(**dict(kw, initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out, ref)
    touched = range(1, len(lengths) + 1)
    for s in touched:
        assert_state_close(pool[s], ref_pool[s], what=f"slot {s}")
    assert_untouched(pool, before, touched)


@pytest.mark.parametrize("heads", (16, 32, 64))
@pytest.mark.parametrize("lengths", [(4,), (4,) * 4, (5,), (1, 2, 3, 4, 5, 6, 7)], ids=str)
def test_decode_checkpoints_match_oracle(ops, heads, lengths):
    """Verify regime: every step checkpointed by batch row, pool untouched."""
    kw = _raw_case(heads, lengths)
    D = 128
    torch.manual_seed(5150)
    noise = (torch.randn(len(lengths), max(lengths), heads, D, D) * 0.1).transpose(-1, -2)
    mid = clone_pool(noise).transpose(-1, -2).to(DEV).transpose(-1, -2)
    dkw = _dev(kw)
    out = ops.kda_varlen_recurrent(**dkw, intermediate_state=mid, prefill=False)
    torch.cuda.synchronize()
    ref_mid = clone_pool(noise)
    ref = kda_ref.kda_varlen_recurrent(**dict(kw, initial_state_source=clone_pool(kw["initial_state_source"])),
                                       intermediate_state=ref_mid, out_fp32=True)
    assert_out_close(out.cpu(), ref)
    got = mid.cpu()
    for r, n in enumerate(lengths):
        assert_state_close(got[r, :n], ref_mid[r, :n], what=f"checkpoints of request {r}")
        assert torch.equal(got[r, n:], noise[r, n:]), "a step past the request's length was written"
    assert torch.equal(dkw["initial_state_source"].cpu(), kw["initial_state_source"])


@pytest.mark.parametrize("lengths", [(4,) * 3, (1, 2, 3, 4, 6), (2, 2)], ids=str)
@pytest.mark.parametrize("log_gate", (False, True))
def test_verify_sized_batches_d64(ops, lengths, log_gate):
    """Verify-sized batches (a few tokens per request, per-step checkpoints)
    at D = 64, with both gate forms."""
    heads, D = 4, 64
    kw = _raw_case(heads, lengths, D=D, seed=17)
    if log_gate:
        T = sum(lengths)
        g = torch.nn.functional.logsigmoid(torch.randn(1, T, heads, D)).clamp(-5.0, 0.0)
        beta = torch.sigmoid(torch.randn(1, T, heads))
        kw = dict(q=kw["q"], k=kw["k"], v=kw["v"], g=g, beta=beta, initial_state_source=kw["initial_state_source"],
                  initial_state_indices=kw["initial_state_indices"], cu_seqlens=kw["cu_seqlens"], scale=kw["scale"])
    noise = (torch.randn(len(lengths), max(lengths), heads, D, D) * 0.1).transpose(-1, -2)
    mid = clone_pool(noise).transpose(-1, -2).to(DEV).transpose(-1, -2)
    dkw = _dev(kw)
    op = ops.kda_varlen_recurrent_g if log_gate else ops.kda_varlen_recurrent
    out = op(**dkw, intermediate_state=mid, prefill=False)
    torch.cuda.synchronize()
    ref_mid = clone_pool(noise)
    ref_fn = kda_ref.kda_varlen_recurrent_g if log_gate else kda_ref.kda_varlen_recurrent
    ref = ref_fn(**dict(kw, initial_state_source=clone_pool(kw["initial_state_source"])),
                 intermediate_state=ref_mid, out_fp32=True)
    assert_out_close(out.cpu(), ref)
    got = mid.cpu()
    for r, n in enumerate(lengths):
        assert_state_close(got[r, :n], ref_mid[r, :n], what=f"checkpoints of request {r}")


def test_cfg2_decode_full_size(ops):
    """BASELINE config 2 at full size: 256 requests, H=32, pool of 512 slots."""
    import kda_workloads as workloads
    w = workloads.config2()
    before = clone_pool(w.pool)
    d = w.to(DEV)
    out = ops.kda_varlen_recurrent_g(**d.kwargs(), prefill=False)
    torch.cuda.synchronize()
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out.cpu(), ref)
    got = d.pool.cpu()
    idx = w.indices.long()
    assert_state_close(got[idx], ref_pool[idx])
    assert_untouched(got, before, idx.tolist())


# ---------------------------------------------------------------------------
# Through the C ABI: fp32 verification output, bit-equal to the torch op
# ---------------------------------------------------------------------------

def test_cfg5_mixed_batch_recurrent(ops):
    """BASELINE config 5 through the recurrent op in its prefill regime (the
    whole mixed batch of 64 one-token and 4 resumed 2048-token requests in one
    call): outputs and updated slots against the oracle, other slots bit-equal."""
    import kda_workloads as workloads
    w = workloads.config5(seed=1)
    before = clone_pool(w.pool)
    d = w.to(DEV)
    out = ops.kda_varlen_recurrent_g(**d.kwargs(), prefill=True)
    torch.cuda.synchronize()
    got = d.pool.cpu()
    del d
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out.cpu(), ref)
    touched = [int(s) for s in w.indices]
    assert_state_close(got[touched], ref_pool[touched])
    assert_untouched(got, before, touched)


def test_abi_fp32_output_meets_bar(abi):
    import kda_workloads as workloads
    w = workloads.config2(requests=64, heads=8, slots=80)
    d = w.to(DEV)
    out32 = torch.empty(d.v.shape, dtype=torch.float32, device=DEV)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out32, state=d.pool, indices=d.indices,
                                 cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                 g=d.g, beta=d.beta, status=status, out_fp32=True)
    assert abi.recurrent_launch(args) == abi.KDA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    ref_pool = clone_pool(w.pool)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=ref_pool), out_fp32=True)
    assert_out_close(out32.cpu(), ref)
    idx = w.indices.long()
    assert_state_close(d.pool.cpu()[idx], ref_pool[idx])


def test_abi_matches_torch_op_bitwise(ops, abi):
    kw = _raw_case(8, (3, 1, 2))
    dkw = _dev(kw)
    pool_a = clone_pool(dkw["initial_state_source"])
    pool_b = clone_pool(dkw["initial_state_source"])
    out_a = ops.kda_varlen_recurrent(**dict(dkw, initial_state_source=pool_a))
    out_b = torch.zeros_like(out_a)
    args = abi.args_from_tensors(q=dkw["q"], k=dkw["k"], v=dkw["v"], out=out_b, state=pool_b,
                                 indices=dkw["initial_state_indices"], cu_seqlens=dkw["cu_seqlens"],
                                 scale=kw["scale"], gate_mode=abi.KDA_GATE_RAW, a=dkw["a"], b=dkw["b"],
                                 A_log=dkw["A_log"], dt_bias=dkw["dt_bias"], lower_bound=kw["lower_bound"])
    assert abi.recurrent_launch(args) == abi.KDA_OK
    torch.cuda.synchronize()
    assert torch.equal(out_a, out_b)
    assert torch.equal(pool_a, pool_b)


def test_abi_reports_bad_slot_without_touching_memory(abi):
    """An out-of-range slot index is caught by the kernel's bounds check."""
    import kda_workloads as workloads
    w = workloads.config2(requests=4, heads=2, slots=8)
    d = w.to(DEV)
    d.indices[2] = 8                                   # one past the pool
    before = clone_pool(d.pool)
    out = torch.zeros_like(d.v)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=d.pool, indices=d.indices,
                                 cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                 g=d.g, beta=d.beta, status=status)
    assert abi.recurrent_launch(args) == abi.KDA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0x102
    touched = [int(s) for i, s in enumerate(d.indices.tolist()) if i != 2]
    assert_untouched(d.pool, before, touched)


@pytest.mark.parametrize("prefill", (False, True))
def test_uncovered_tokens_read_zero(ops, prefill):
    """The op returns zeros wherever it computes nothing, as the reference's
    zeros_like output does (kda_varlen_recurrent.cpp:142): tokens before
    cu_seqlens[0] and after cu_seqlens[-1]. The output memory is dirtied first
    so a missing write cannot pass by the allocator's luck."""
    kw = _raw_case(3, (3, 4), slots=6, seed=8)
    tokens = 12
    for n in ("q", "k", "v", "a"):
        kw[n] = (torch.randn(1, tokens, 3, 128) * 0.2).bfloat16()
    kw["b"] = torch.randn(1, tokens, 3).bfloat16()
    kw["cu_seqlens"] = torch.tensor([2, 5, 9], dtype=torch.int32)
    ref_kw = dict(kw)
    ref_pool = clone_pool(kw["initial_state_source"])
    ref = kda_ref.kda_varlen_recurrent(**dict(ref_kw, initial_state_source=ref_pool), out_fp32=True,
                                       prefill=prefill)
    for _ in range(3):                                 # leave non-zero bytes in the allocator's blocks
        junk = torch.full((1, tokens, 3, 128), 7.0, dtype=torch.bfloat16, device=DEV)
        del junk
    out, pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=prefill)
    assert torch.equal(out[:, :2], torch.zeros_like(out[:, :2]))
    assert torch.equal(out[:, 9:], torch.zeros_like(out[:, 9:]))
    assert_out_close(out[:, 2:9], ref[:, 2:9])
    assert_state_close(pool[1:3], ref_pool[1:3])


def test_rejected_request_rows_read_zero(abi):
    """A request whose slot fails the bounds check computes nothing: its
    output rows are zeros (the C ABI writes every token), the others match."""
    import kda_workloads as workloads
    w = workloads.config2(requests=4, heads=2, slots=8)
    d = w.to(DEV)
    d.indices[1] = 8                                   # one past the pool
    out = torch.full_like(d.v, 7.0)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    args = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=d.pool, indices=d.indices,
                                 cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                 g=d.g, beta=d.beta, status=status)
    assert abi.recurrent_launch(args) == abi.KDA_OK
    torch.cuda.synchronize()
    assert int(status.item()) == 0x102
    assert torch.equal(out[:, 1], torch.zeros_like(out[:, 1]))
    assert (out[:, [0, 2, 3]] != 7.0).all()


# ---------------------------------------------------------------------------
# Index dtypes (test_kda_index_dtypes.py:69-103): bit-exact
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("index_dtype,starts_dtype",
                         [p for p in itertools.product((torch.int32, torch.int64), repeat=2)
                          if p != (torch.int32, torch.int32)])
def test_index_dtype_does_not_change_result(ops, index_dtype, starts_dtype):
    base = _raw_case(4, (257,), slots=6, seed=5)
    base["initial_state_indices"] = torch.tensor([3], dtype=torch.int32)
    out_a, pool_a = _run_op(ops.kda_varlen_recurrent, base, prefill=True)
    kw = dict(base, initial_state_indices=base["initial_state_indices"].to(index_dtype),
              cu_seqlens=base["cu_seqlens"].to(starts_dtype))
    out_b, pool_b = _run_op(ops.kda_varlen_recurrent, kw, prefill=True)
    assert out_b.float().abs().sum() > 0, "op returned its zeroed output"
    assert torch.equal(out_a, out_b)
    assert torch.equal(pool_a, pool_b)


@pytest.mark.parametrize("track_dtype", (torch.int32, torch.int64))
def test_track_dtype_does_not_change_checkpoint(ops, track_dtype):
    base = _raw_case(4, (257,), slots=6, seed=5)
    base["initial_state_indices"] = torch.tensor([3], dtype=torch.int32)
    t32 = dict(track_state_indices=torch.tensor([5], dtype=torch.int32).to(DEV),
               track_state_lens=torch.tensor([64], dtype=torch.int32).to(DEV))
    out_a, pool_a = _run_op(ops.kda_varlen_recurrent, base, prefill=True, **t32)
    tx = {k: v.to(track_dtype) for k, v in t32.items()}
    out_b, pool_b = _run_op(ops.kda_varlen_recurrent, base, prefill=True, **tx)
    assert torch.equal(out_a, out_b)
    assert torch.equal(pool_a, pool_b)
    assert pool_b[5].abs().sum() > 0, "checkpoint slot unwritten"


# ---------------------------------------------------------------------------
# Prefix tracking and resume (test_glm53_kda_prefix_ascendc.py:97-182)
# ---------------------------------------------------------------------------

@pytest.mark.parametrize("cut", [0, 1, 63, 64, 100, 129])
def test_prefix_checkpoint_and_resume(ops, cut):
    lengths = (129, 65, 63)
    kw = _raw_case(4, lengths, slots=12, seed=cut)
    kw["initial_state_indices"] = torch.tensor([3, 1, 5], dtype=torch.int64)
    dests = torch.tensor([9, 7, 0], dtype=torch.int64)
    cuts = torch.tensor([min(cut, n) for n in lengths], dtype=torch.int32)
    base_out, base_pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=True)
    tr_out, tr_pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=True,
                              track_state_indices=dests.to(DEV), track_state_lens=cuts.to(DEV))
    assert torch.equal(tr_out, base_out)
    for s in (3, 1, 5):
        assert torch.equal(tr_pool[s], base_pool[s])
    ref_pool = clone_pool(kw["initial_state_source"])
    kda_ref.kda_varlen_recurrent(**dict(kw, initial_state_source=ref_pool), track_state_indices=dests,
                                 track_state_lens=cuts)
    for d in (9, 7):
        assert_state_close(tr_pool[d], ref_pool[d], tol=2e-4, what=f"checkpoint slot {d}")
    assert_untouched(tr_pool, kw["initial_state_source"], {3, 1, 5, 9, 7})
    # Resume the first request from its checkpoint: same final state and tail.
    n0, c0 = lengths[0], int(cuts[0])
    if c0 < n0:
        resumed = dict(kw)
        sl = slice(c0, n0)
        for name in ("q", "k", "v", "a", "b"):
            resumed[name] = kw[name][:, sl].contiguous()
        pool = clone_pool(kw["initial_state_source"])
        pool[3] = tr_pool[9]
        resumed["initial_state_source"] = pool
        resumed["initial_state_indices"] = torch.tensor([3], dtype=torch.int32)
        resumed["cu_seqlens"] = torch.tensor([0, n0 - c0], dtype=torch.int32)
        out, pool_after = _run_op(ops.kda_varlen_recurrent, resumed, prefill=True)
        assert_out_close(out, base_out[:, sl].float(), tol=2e-2)
        assert state_error(pool_after[3], base_pool[3]) <= 2e-4


# ---------------------------------------------------------------------------
# CUDA graph: capture once, replay with changed metadata behind the pointers
# (test_glm53_kda_prefix_ascendc.py:185-293)
# ---------------------------------------------------------------------------

def test_cuda_graph_replay_with_changed_metadata(ops):
    heads, D, batch, steps = 4, 128, 6, 2
    kw = _raw_case(heads, (steps,) * batch, slots=2 * batch + 3, seed=7)
    dkw = _dev(kw)
    initial = clone_pool(dkw["initial_state_source"])
    work = dkw["initial_state_source"]
    slots = dkw["initial_state_indices"]
    for _ in range(3):
        work.copy_(initial)
        ops.kda_varlen_recurrent(**dkw, prefill=False)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        with torch.cuda.graph(graph):
            captured = ops.kda_varlen_recurrent(**dkw, prefill=False)
    torch.cuda.synchronize()
    for replay in range(4):
        active = [(row + replay) % (batch + 1) for row in range(batch)]
        slots.copy_(torch.tensor(active, dtype=slots.dtype))
        for name in ("q", "k", "v", "a"):
            dkw[name].copy_((torch.randn_like(dkw[name].float()) * 0.2).bfloat16())
        work.copy_(initial)
        ref_pool = clone_pool(initial)
        expected = ops.kda_varlen_recurrent(**dict(dkw, initial_state_source=ref_pool), prefill=False)
        torch.cuda.synchronize()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(work, ref_pool)
        assert torch.equal(captured, expected)
    del graph


# ---------------------------------------------------------------------------
# Rejections the caller matches on (test_kda.py:290-332)
# ---------------------------------------------------------------------------

def test_rejects_transposed_state(ops):
    kw = _dev(_raw_case(8, (128,)))
    kw["initial_state_source"] = kw["initial_state_source"].transpose(-1, -2)
    with pytest.raises(RuntimeError, match="K-contiguous"):
        ops.kda_varlen_recurrent(**kw, prefill=True)


def test_rejects_prefill_intermediate_state(ops):
    kw = _dev(_raw_case(8, (16,)))
    mid = torch.zeros(1, 16, 8, 128, 128, device=DEV).transpose(-1, -2)
    with pytest.raises(RuntimeError, match="does not support intermediate_state"):
        ops.kda_varlen_recurrent(**kw, intermediate_state=mid, prefill=True)


def test_rejects_transposed_intermediate_state(ops):
    kw = _dev(_raw_case(16, (4,) * 3))
    mid = torch.zeros(3, 4, 16, 128, 128, device=DEV)
    with pytest.raises(RuntimeError, match="K-contiguous"):
        ops.kda_varlen_recurrent(**kw, intermediate_state=mid, prefill=False)


def test_rejects_fewer_tokens_than_requests(ops):
    kw = _dev(_raw_case(16, (1, 1, 0)))
    with pytest.raises(RuntimeError, match="one token per request"):
        ops.kda_varlen_recurrent(**kw, prefill=False)


def test_any_head_count_and_multi_sequence_prefill(ops):
    """The reference rejects these (test_kda.py:252-274); the B200 op serves them."""
    for heads, lengths, prefill in [(2, (128,), True), (16, (128,), True), (8, (1,) * 3, False),
                                    (8, (128, 128), True)]:
        kw = _raw_case(heads, lengths)
        out, pool = _run_op(ops.kda_varlen_recurrent, kw, prefill=prefill)
        ref = kda_ref.kda_varlen_recurrent(**dict(kw, initial_state_source=clone_pool(kw["initial_state_source"])),
                                           out_fp32=True)
        assert_out_close(out, ref)
