"""The reference's backend checkpoint contract, with the implementation pluggable.

``check_backend`` in
``sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387``
runs sglang's extend step (causal conv over the mixed q | k | v projection,
then the KDA op) three ways on a 513-token request that continues a 512-token
prefix -- whole, whole with a tracked-prefix checkpoint at token 256, and only
the first 256 tokens -- and resumes a fourth run from the checkpoint. Its
assertions (reproduced by :func:`check_contract`, same tolerances):

* the tracked run's output and final states equal the untracked run's,
  bit for bit;
* the temporal checkpoint equals the prefix run's final state (rtol 2e-4,
  atol 2e-5); the conv checkpoint is the ``window`` raw rows before the cut,
  and its last 3 rows are the prefix run's final conv rows;
* the resumed suffix reproduces the whole run's tail (rtol 8e-3, atol 1e-3)
  and its final states (temporal 2e-4 / 2e-5, conv last rows exact);
* every other slot of both pools is untouched.

``impl(mixed, a, b, layer, conv, temporal, idx, cu, has_init, tidx, tlen)``
runs one extend call and returns its output [1, T, H, D]; it updates
``conv`` ([slots, window, C] bf16) and ``temporal`` ([slots, H, K, V] fp32,
K-contiguous) in place. Inputs are seeded synthetic ones of the reference's
shapes (4 heads of 128, 4 taps, 10 slots).
"""

from __future__ import annotations

from types import SimpleNamespace

import torch

TOTAL, CUT, SOURCE, DESTINATION, SLOTS, HEADS, D = 513, 256, 3, 7, 10, 4, 128


def make_inputs(window: int, device="cpu"):
    g = torch.Generator().manual_seed(20260915 + window)
    C = 3 * HEADS * D

    def rnd(*shape, s=1.0):
        return torch.randn(*shape, generator=g) * s

    layer = SimpleNamespace(conv_weights=rnd(C, 4, s=0.1), A_log=rnd(HEADS, s=0.1),
                            dt_bias=rnd(HEADS * D, s=0.1), lower_bound=-5.0)
    ins = SimpleNamespace(
        conv_seed=rnd(SLOTS, window, C, s=0.1).bfloat16(),
        temporal_seed=rnd(SLOTS, HEADS, D, D, s=0.1),
        mixed=rnd(TOTAL, C, s=0.2).bfloat16(),
        a=rnd(1, TOTAL, HEADS * D, s=0.2).bfloat16(),
        b=rnd(1, TOTAL, HEADS).bfloat16(),
        layer=layer, window=window)
    if device != "cpu":
        for k, v in list(vars(ins).items()):
            if torch.is_tensor(v):
                setattr(ins, k, v.to(device))
        for k, v in list(vars(layer).items()):
            if torch.is_tensor(v):
                setattr(layer, k, v.to(device))
    return ins


def _kcontig(t: torch.Tensor) -> torch.Tensor:
    return t.transpose(-1, -2).contiguous().transpose(-1, -2)


def new_cache(ins):
    return SimpleNamespace(conv=ins.conv_seed.clone(), temporal=_kcontig(ins.temporal_seed))


def run(impl, ins, cache, begin, end, tracking):
    dev = ins.mixed.device
    i32 = dict(dtype=torch.int32, device=dev)
    idx = torch.tensor([SOURCE], **i32)
    cu = torch.tensor([0, end - begin], **i32)
    has_init = torch.tensor([True], device=dev)        # the request continues a 512 + begin token prefix
    tidx = torch.tensor([DESTINATION], **i32) if tracking else None
    tlen = torch.tensor([CUT - begin], **i32) if tracking else None
    return impl(ins.mixed[begin:end], ins.a[:, begin:end], ins.b[:, begin:end], ins.layer,
                cache.conv, cache.temporal, idx, cu, has_init, tidx, tlen)


def check_contract(impl, ins) -> dict:
    window = ins.window
    baseline, tracked, prefix = new_cache(ins), new_cache(ins), new_cache(ins)
    expected = run(impl, ins, baseline, 0, TOTAL, False)
    actual = run(impl, ins, tracked, 0, TOTAL, True)
    run(impl, ins, prefix, 0, CUT, False)
    cpu = lambda t: t.detach().cpu()  # noqa: E731
    assert torch.equal(cpu(actual), cpu(expected)), "tracked run's output differs from the untracked run's"
    assert torch.equal(cpu(tracked.temporal[SOURCE]), cpu(baseline.temporal[SOURCE]))
    torch.testing.assert_close(cpu(tracked.temporal[DESTINATION]), cpu(prefix.temporal[SOURCE]),
                               rtol=2e-4, atol=2e-5)
    assert torch.equal(cpu(tracked.conv[DESTINATION]), cpu(ins.mixed[CUT - window:CUT]))
    assert torch.equal(cpu(tracked.conv[DESTINATION, -3:]), cpu(prefix.conv[SOURCE, -3:]))
    resumed = new_cache(ins)
    resumed.temporal[SOURCE] = tracked.temporal[DESTINATION]
    resumed.conv[SOURCE] = tracked.conv[DESTINATION]
    suffix = run(impl, ins, resumed, CUT, TOTAL, False)
    torch.testing.assert_close(cpu(suffix).float(), cpu(expected[:, CUT:]).float(), rtol=0.008, atol=0.001)
    torch.testing.assert_close(cpu(resumed.temporal[SOURCE]), cpu(baseline.temporal[SOURCE]), rtol=2e-4, atol=2e-5)
    assert torch.equal(cpu(resumed.conv[SOURCE, -3:]), cpu(baseline.conv[SOURCE, -3:]))
    for slot in set(range(SLOTS)) - {SOURCE, DESTINATION}:
        assert torch.equal(cpu(tracked.temporal[slot]), cpu(ins.temporal_seed[slot]))
        assert torch.equal(cpu(tracked.conv[slot]), cpu(ins.conv_seed[slot]))
    return dict(expected=expected, checkpoint=tracked.temporal[DESTINATION].clone(),
                conv_checkpoint=tracked.conv[DESTINATION].clone(), final_conv=baseline.conv[SOURCE].clone())


def oracle_impl(mixed, a, b, layer, conv, temporal, idx, cu, has_init, tidx, tlen):
    """The extend step on the CPU oracles (conv, then the chunked KDA op)."""
    from oracle import conv_ref, kda_ref

    planes, status = conv_ref.causal_conv1d(mixed, layer.conv_weights, None, conv, idx, cu, has_init,
                                            tidx, tlen, activation="silu", num_parts=3)
    assert status == 0
    T = mixed.shape[0]
    q, k, v = (planes[i].view(1, T, HEADS, D) for i in range(3))
    return kda_ref.kda_varlen_chunk(
        A_log=layer.A_log, a=a.reshape(1, T, HEADS, D), dt_bias=layer.dt_bias, q=q, k=k, v=v,
        b=b.reshape(1, T, HEADS), initial_state_source=temporal, initial_state_indices=idx, cu_seqlens=cu,
        lower_bound=layer.lower_bound, scale=D ** -0.5, track_state_indices=tidx, track_state_lens=tlen)


def oracle_decode_impl(mixed, a, b, layer, conv, temporal, idx, cu):
    """The decode step on the CPU oracles (conv, then the token recurrence)."""
    from oracle import conv_ref, kda_ref

    planes, status = conv_ref.causal_conv1d(mixed, layer.conv_weights, None, conv, idx, cu,
                                            activation="silu", num_parts=3)
    assert status == 0
    T = mixed.shape[0]
    q, k, v = (planes[i].view(1, T, HEADS, D) for i in range(3))
    return kda_ref.kda_varlen_recurrent(
        A_log=layer.A_log, a=a.reshape(1, T, HEADS, D), dt_bias=layer.dt_bias, q=q, k=k, v=v,
        b=b.reshape(1, T, HEADS), initial_state_source=temporal, initial_state_indices=idx, cu_seqlens=cu,
        lower_bound=layer.lower_bound, scale=D ** -0.5, prefill=False)


PREFIX_LENS = (20, 7, 33)
DECODE_STEPS = 3
DECODE_SLOTS = (2, 5, 8)


def decode_continuation(extend_impl, decode_impl, ins) -> dict:
    """Extend three requests over their prefixes, then decode DECODE_STEPS
    tokens of each, one batched step at a time; against one extend over the
    whole sequences. Both runs start from the same pools; returns the decode
    outputs and final pools of both."""
    dev = ins.mixed.device
    i32 = dict(dtype=torch.int32, device=dev)
    R = len(PREFIX_LENS)
    full_lens = [n + DECODE_STEPS for n in PREFIX_LENS]
    # token rows: request r's tokens are rows starts[r] .. starts[r] + full_lens[r]
    starts = [0]
    for n in full_lens[:-1]:
        starts.append(starts[-1] + n)
    idx = torch.tensor(DECODE_SLOTS, **i32)
    init = torch.ones(R, dtype=torch.bool, device=dev)

    def rows(pick):
        sel = torch.cat([torch.arange(s + lo, s + hi) for s, (lo, hi) in zip(starts, pick)]).to(dev)
        cu = [0]
        for lo, hi in pick:
            cu.append(cu[-1] + hi - lo)
        return sel, torch.tensor(cu, **i32)

    def take(sel):
        return ins.mixed[sel], ins.a[:, sel], ins.b[:, sel]

    whole = new_cache(ins)
    sel, cu = rows([(0, n) for n in full_lens])
    out_whole = extend_impl(*take(sel), ins.layer, whole.conv, whole.temporal, idx, cu, init, None, None)
    stepped = new_cache(ins)
    sel, cu = rows([(0, n) for n in PREFIX_LENS])
    extend_impl(*take(sel), ins.layer, stepped.conv, stepped.temporal, idx, cu, init, None, None)
    outs = []
    for step in range(DECODE_STEPS):
        sel, cu = rows([(n + step, n + step + 1) for n in PREFIX_LENS])
        outs.append(decode_impl(*take(sel), ins.layer, stepped.conv, stepped.temporal, idx, cu))
    # the whole run's outputs at the decoded positions, in step order
    want = []
    for step in range(DECODE_STEPS):
        pos = [sum(full_lens[:r]) + PREFIX_LENS[r] + step for r in range(R)]
        want.append(out_whole[:, pos])
    return dict(decoded=torch.stack(outs), whole=torch.stack(want), stepped=stepped, whole_cache=whole)


def check_decode_continuation(extend_impl, decode_impl, ins) -> dict:
    r = decode_continuation(extend_impl, decode_impl, ins)
    cpu = lambda t: t.detach().cpu()  # noqa: E731
    torch.testing.assert_close(cpu(r["decoded"]).float(), cpu(r["whole"]).float(), rtol=0.008, atol=0.001)
    for s in DECODE_SLOTS:
        torch.testing.assert_close(cpu(r["stepped"].temporal[s]), cpu(r["whole_cache"].temporal[s]),
                                   rtol=2e-4, atol=2e-5)
        assert torch.equal(cpu(r["stepped"].conv[s]), cpu(r["whole_cache"].conv[s]))
    for s in set(range(SLOTS)) - set(DECODE_SLOTS):
        assert torch.equal(cpu(r["stepped"].conv[s]), cpu(ins.conv_seed[s]))
        assert torch.equal(cpu(r["stepped"].temporal[s]), cpu(ins.temporal_seed[s]))
    return r
