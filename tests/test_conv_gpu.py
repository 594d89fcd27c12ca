"""GPU parity of the causal-conv front end (``kda_causal_conv1d`` / ``kda_conv_launch``).

Against ``oracle/conv_ref.py`` on the same seeded inputs:

* outputs within one bf16 ulp of the oracle's fp32 pre-cast values plus an
  absolute 2^-20 (the kernel sums the taps with fused multiply-adds, the
  oracle rounds each product, so the fp32 sums differ by ~1e-8; that only
  shows where the taps cancel to a result near zero), and almost all of them
  equal to the oracle's own bf16 rounding;
* conv-state rows and checkpoints bit-exact (they are copies of input rows);
* untouched slots (and the padding slot 0) bit-identical;
* rejected requests: status word, zero output rows, nothing written.

Batches cover long requests (16-token streaming tiles, requests starting at
a tile's last token), short mixed requests and a decode batch (all work in
the per-request CTAs), empty and one-token requests, fresh and continuing
requests, checkpoints at 0, inside and at the end of a request, row strides
wider than the channel count, and the reference's backend checkpoint
contract through ``kda_forward_extend`` (conv, then the chunked KDA op), and
decode steps through ``kda_forward_decode`` (conv, then the token recurrence)
continuing an extend as one longer extend would, against the oracles.
"""

import pytest
import torch

import conv_backend
from kda_checks import assert_out_close, assert_state_close
from oracle import conv_ref

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def ops():
    import sgl_glm53_ascend_ops  # noqa: F401  (loads the op library)
    from sgl_glm53_ascend_ops import ops as _ops
    return _ops


@pytest.fixture
def status():
    buf = torch.zeros(1, dtype=torch.int32, device=DEV)
    torch.ops.sgl_glm53_ascend.kda_set_status_buffer(0, buf)
    yield buf
    torch.ops.sgl_glm53_ascend.kda_set_status_buffer(0, None)


def _ulp(ref: torch.Tensor) -> torch.Tensor:
    return torch.ldexp(torch.ones_like(ref), torch.frexp(ref)[1] - 8)


def _batch(lengths, C, window, W=4, slots=None, seed=0, init_every=2, track=None, bias=True, wide=0,
           idx_dtype=torch.int32):
    g = torch.Generator().manual_seed(seed)
    R = len(lengths)
    slots = slots or (2 * R + 3)
    T = sum(lengths)
    x_full = (torch.randn(T, C + wide, generator=g) * 0.5).bfloat16()
    x = x_full[:, :C]
    weight = torch.randn(C, W, generator=g) * 0.3
    b = torch.randn(C, generator=g) * 0.1 if bias else None
    state = (torch.randn(slots, window, C, generator=g) * 0.5).bfloat16()
    perm = torch.randperm(slots - 1, generator=g) + 1
    idx = perm[:R].to(idx_dtype)
    cu = torch.tensor([0] + torch.tensor(lengths).cumsum(0).tolist(), dtype=idx_dtype)
    init = torch.tensor([(i % init_every) != 0 for i in range(R)])
    tidx = tlen = None
    if track is not None:
        tidx = torch.zeros(R, dtype=idx_dtype)
        tlen = torch.zeros(R, dtype=idx_dtype)
        for i, (r, n) in enumerate(track):
            tidx[r] = int(perm[R + i])
            tlen[r] = n
    return dict(x=x, x_full=x_full, weight=weight, bias=b, state=state, idx=idx, cu=cu, init=init,
                tidx=tidx, tlen=tlen)


def _dev(t):
    return None if t is None else t.to(DEV)


def _run_gpu(b, num_parts=3, silu=True):
    x = b["x_full"].to(DEV)[:, :b["x"].shape[1]]
    st = b["state"].to(DEV)
    out = torch.ops.sgl_glm53_ascend.kda_causal_conv1d(
        x, _dev(b["weight"]), _dev(b["bias"]), st, _dev(b["idx"]), _dev(b["cu"]), _dev(b["init"]),
        _dev(b["tidx"]), _dev(b["tlen"]), num_parts, silu)
    torch.cuda.synchronize()
    return out.cpu(), st.cpu()


def _run_oracle(b, num_parts=3, silu=True):
    st = b["state"].clone()
    out32, status = conv_ref.causal_conv1d(b["x"], b["weight"], b["bias"], st, b["idx"], b["cu"], b["init"],
                                           b["tidx"], b["tlen"], activation="silu" if silu else None,
                                           num_parts=num_parts, out_fp32=True)
    return out32, st, status


def _check(b, num_parts=3, silu=True):
    out, st = _run_gpu(b, num_parts, silu)
    ref32, ref_st, ref_status = _run_oracle(b, num_parts, silu)
    assert ref_status == 0
    d = (out.float() - ref32).abs() - _ulp(ref32)
    assert bool((d <= 2.0 ** -20).all()), f"output more than one bf16 ulp from the oracle ({d.max():.3e} over)"
    exact = (out == ref32.bfloat16()).float().mean().item() if out.numel() else 1.0
    assert exact >= 0.99, f"only {exact:.4f} of the outputs equal the oracle's bf16 rounding"
    assert torch.equal(st, ref_st), "conv state differs from the oracle (touched or untouched slots)"
    return out, st


@pytest.mark.parametrize("window", [3, 6])
def test_prefill_tiles_of_16(window):
    # requests start at a tile's last token (15, 31, ...) and straddle tiles
    lengths = [15, 1, 16, 40, 0, 3, 100, 17, 2, 64]
    b = _batch(lengths, C=1536, window=window, track=[(3, 0), (6, 37), (9, 64), (7, 18)])
    _check(b)


def test_mixed_short_requests():
    lengths = [1, 1, 3, 4, 7, 2, 0, 9, 1, 5, 13, 2, 1, 6]
    b = _batch(lengths, C=3 * 2 * 128, window=4, seed=1, init_every=3, track=[(4, 3), (10, 12)])
    _check(b)


def test_decode_batch():
    # BASELINE config 2's decode shape: 256 one-token requests, H = 32 heads of q | k | v
    b = _batch([1] * 256, C=3 * 32 * 128, window=3, seed=2)
    b["init"] = torch.ones(256, dtype=torch.bool)
    _check(b)


@pytest.mark.parametrize("W", [1, 2, 3])
def test_fewer_taps_no_activation(W):
    b = _batch([5, 20, 1, 33], C=256, window=max(W - 1, 1) + 1, W=W, seed=3 + W, bias=False)
    _check(b, num_parts=1, silu=False)


def test_wide_rows_int64_indices_int_flags():
    b = _batch([7, 30, 2, 19], C=768, window=3, seed=7, wide=136, idx_dtype=torch.int64,
               track=[(1, 29), (3, 19)])
    b["init"] = b["init"].to(torch.int32)
    _check(b)


def test_padding_slot_and_empty_batch_checkpoint(status):
    b = _batch([4, 6], C=256, window=3, seed=9, track=[(0, 2)])
    b["idx"][1] = 0                                           # request 1 on the padding slot
    out, st = _check(b, num_parts=1)
    assert torch.equal(st[0], b["state"][0])
    assert status.item() == 0
    # no tokens at all: a checkpoint at length 0 still copies the old window
    e = _batch([0, 0], C=256, window=3, seed=10, track=[(1, 0)])
    _check(e, num_parts=1)


@pytest.mark.parametrize("lengths", [[1] * 8, [10, 20, 7]])
def test_uncovered_rows_read_zero(lengths):
    """Tokens before the first request and after the last one get zero rows,
    in a batch of short requests (one launch) and of longer ones (two)."""
    b = _batch(lengths, C=768, window=3, seed=13)
    lead, tail = 3, 5
    T = sum(lengths) + lead + tail
    g = torch.Generator().manual_seed(14)
    b["x_full"] = (torch.randn(T, 768, generator=g) * 0.5).bfloat16()
    b["x"] = b["x_full"]
    b["cu"] = b["cu"] + lead
    out, st = _check(b)
    assert torch.equal(out[:, :lead], torch.zeros_like(out[:, :lead]))
    assert torch.equal(out[:, T - tail:], torch.zeros_like(out[:, T - tail:]))


def test_no_requests_zero_every_row():
    x = torch.randn(5, 768, device=DEV).bfloat16()
    w = torch.randn(768, 4, device=DEV)
    st = torch.randn(3, 3, 768, device=DEV).bfloat16()
    before = st.clone()
    out = torch.ops.sgl_glm53_ascend.kda_causal_conv1d(
        x, w, None, st, torch.zeros(0, dtype=torch.int32, device=DEV), torch.zeros(1, dtype=torch.int32, device=DEV),
        None, None, None, 3, True)
    torch.cuda.synchronize()
    assert out.shape == (3, 5, 256) and not bool(out.any())
    assert torch.equal(st, before)


@pytest.mark.parametrize("lengths", [[5, 9, 3], [1, 2, 1]])
def test_rejected_requests(status, lengths):
    b = _batch(lengths, C=256, window=3, seed=11)
    b["idx"][1] = 10 ** 6                                     # slot out of range
    out, st = _run_gpu(b, num_parts=1)
    assert status.item() == conv_ref.BAD_SLOT
    ref32, ref_st, ref_status = _run_oracle(b, num_parts=1)
    assert ref_status == conv_ref.BAD_SLOT
    lo, hi = lengths[0], lengths[0] + lengths[1]
    assert torch.equal(out[0, lo:hi], torch.zeros(hi - lo, 256, dtype=torch.bfloat16))
    keep = torch.ones(out.shape[1], dtype=torch.bool)
    keep[lo:hi] = False
    d = (out[0, keep].float() - ref32[0, keep]).abs() - _ulp(ref32[0, keep])
    assert bool((d <= 2.0 ** -20).all())
    assert torch.equal(st, ref_st)


def test_c_abi_matches_torch_op():
    from sgl_glm53_ascend_ops import abi

    b = _batch([3, 50, 1, 21], C=1536, window=6, seed=12, track=[(1, 17)])
    out_op, st_op = _run_gpu(b)
    x = b["x"].to(DEV)
    st = b["state"].to(DEV)
    out = torch.empty(3, x.shape[0], 512, dtype=torch.bfloat16, device=DEV)
    args = abi.conv_args_from_tensors(
        x=x, weight=b["weight"].to(DEV), bias=_dev(b["bias"]), conv_state=st, indices=_dev(b["idx"]),
        cu_seqlens=_dev(b["cu"]), out=out, has_initial=_dev(b["init"]), track_indices=_dev(b["tidx"]),
        track_lens=_dev(b["tlen"]))
    assert abi.conv_launch(args) == abi.KDA_OK
    torch.cuda.synchronize()
    assert torch.equal(out.cpu(), out_op)
    assert torch.equal(st.cpu(), st_op)


def _gpu_impl(ops):
    def impl(mixed, a, b, layer, conv, temporal, idx, cu, has_init, tidx, tlen):
        return ops.kda_forward_extend(
            mixed=mixed, a=a, b=b, conv_weights=layer.conv_weights, conv_bias=None, A_log=layer.A_log,
            dt_bias=layer.dt_bias, lower_bound=layer.lower_bound, conv_state=conv, temporal_state=temporal,
            cache_indices=idx, query_start_loc=cu, head_dim=conv_backend.D, has_initial_state=has_init,
            track_indices=tidx, track_lens=tlen)
    return impl


@pytest.mark.parametrize("window", [3, 6])
def test_backend_checkpoint_contract_on_gpu(ops, window):
    """The reference's check_backend assertions on the B200 extend step, and
    its results against the oracle composition."""
    got = conv_backend.check_contract(_gpu_impl(ops), conv_backend.make_inputs(window, device=DEV))
    ref = conv_backend.check_contract(conv_backend.oracle_impl, conv_backend.make_inputs(window))
    assert_out_close(got["expected"], ref["expected"], what="extend output")
    assert_state_close(got["checkpoint"], ref["checkpoint"], what="temporal checkpoint")
    assert torch.equal(got["conv_checkpoint"].cpu(), ref["conv_checkpoint"])
    assert torch.equal(got["final_conv"].cpu(), ref["final_conv"])


def _gpu_decode_impl(ops):
    def impl(mixed, a, b, layer, conv, temporal, idx, cu):
        return ops.kda_forward_decode(
            mixed=mixed, a=a, b=b, conv_weights=layer.conv_weights, conv_bias=None, A_log=layer.A_log,
            dt_bias=layer.dt_bias, lower_bound=layer.lower_bound, conv_state=conv, temporal_state=temporal,
            cache_indices=idx, query_start_loc=cu, head_dim=conv_backend.D)
    return impl


def test_decode_continues_extend_on_gpu(ops):
    """Prefixes through kda_forward_extend, then three batched one-token steps
    through kda_forward_decode: the same outputs and pools as one longer
    extend, and as the oracles' run of the same steps."""
    got = conv_backend.check_decode_continuation(_gpu_impl(ops), _gpu_decode_impl(ops),
                                                 conv_backend.make_inputs(3, device=DEV))
    ref = conv_backend.decode_continuation(conv_backend.oracle_impl, conv_backend.oracle_decode_impl,
                                           conv_backend.make_inputs(3))
    assert_out_close(got["decoded"], ref["decoded"], what="decode outputs")
    for s in conv_backend.DECODE_SLOTS:
        assert_state_close(got["stepped"].temporal[s], ref["stepped"].temporal[s], what=f"temporal slot {s}")
        assert torch.equal(got["stepped"].conv[s].cpu(), ref["stepped"].conv[s])
