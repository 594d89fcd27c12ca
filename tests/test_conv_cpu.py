"""CPU checks of the causal-conv front end's oracle (``oracle/conv_ref.py``).

* Pinned to a published causal conv1d: the fixtures under ``tests/golden/``
  hold vLLM 0.22's ``causal_conv1d_torch`` on seeded inputs
  (``tests/golden/make_conv_golden.py``). The conv itself (no activation,
  one rounding) must match bit for bit, and so must every conv-state row.
  With SiLU vLLM rounds the conv to bf16 before the activation; applying
  torch's SiLU to the oracle's rounded conv reproduces vLLM exactly, and the
  oracle's single-rounding SiLU stays within one bf16 ulp of it.
* The reference's backend checkpoint contract
  (test_glm53_kda_prefix_ascendc.py:325-387, via ``tests/conv_backend.py``)
  holds for the oracle composition conv -> chunked KDA, windows 3 and 6.
* Decode continuation: extending prefixes and then decoding one token per
  request at a time (conv, then the token recurrence) reproduces one extend
  over the whole sequences (the backend's suffix tolerances).
* State rules: padding slot 0, requests that start fresh, empty requests, a
  checkpoint at length 0, rejected slots.
"""

import pytest
import torch
import torch.nn.functional as F

import conv_backend
from golden_io import bf16, load
from oracle import conv_ref

CASES = ("conv_vllm_linear", "conv_vllm_silu", "conv_vllm_w3")


def _run_fixture(f, activation):
    st = bf16(f["state_in"]).clone()
    out, status = conv_ref.causal_conv1d(
        bf16(f["x"]), torch.from_numpy(f["weight"]),
        torch.from_numpy(f["bias"]) if "bias" in f else None, st,
        torch.from_numpy(f["indices"]), torch.from_numpy(f["cu_seqlens"]),
        torch.from_numpy(f["has_initial"]), activation=activation)
    assert status == 0
    return out[0], st


@pytest.mark.parametrize("name", CASES)
def test_oracle_matches_vllm_causal_conv1d(name):
    f = load(name)
    act = str(f["activation"])
    ref = bf16(f["out"])
    conv, st = _run_fixture(f, None)
    assert torch.equal(st, bf16(f["state_out"])), "conv state rows differ"
    if act == "none":
        assert torch.equal(conv, ref)
        return
    # vLLM: SiLU on the bf16-rounded conv (torch computes it in fp32 and rounds)
    assert torch.equal(F.silu(conv), ref)
    one_rounding, _ = _run_fixture(f, "silu")
    d = (one_rounding.float() - ref.float()).abs()
    ulp = torch.ldexp(torch.ones_like(ref.float()), torch.frexp(ref.float())[1] - 8)
    assert bool((d <= ulp).all()), "single-rounding SiLU more than one bf16 ulp from vLLM"


@pytest.mark.parametrize("window", [3, 6])
def test_oracle_meets_backend_checkpoint_contract(window):
    conv_backend.check_contract(conv_backend.oracle_impl, conv_backend.make_inputs(window))


def test_oracle_decode_continues_extend():
    conv_backend.check_decode_continuation(conv_backend.oracle_impl, conv_backend.oracle_decode_impl,
                                           conv_backend.make_inputs(3))


def _small(window=4, W=4, C=16, slots=6, seed=3):
    g = torch.Generator().manual_seed(seed)
    return dict(weight=torch.randn(C, W, generator=g), bias=torch.randn(C, generator=g),
                state=(torch.randn(slots, window, C, generator=g)).bfloat16(), g=g, C=C)


def test_oracle_state_rules():
    s = _small()
    lengths = [3, 0, 1, 6, 2]
    x = torch.randn(sum(lengths), s["C"], generator=s["g"]).bfloat16()
    cu = torch.tensor([0, 3, 3, 4, 10, 12])
    idx = torch.tensor([1, 2, 0, 3, 4])                 # request 2 is on the padding slot
    init = torch.tensor([True, True, True, False, True])
    tidx = torch.tensor([5, 0, 0, 0, 0])
    tlen = torch.tensor([0, 0, 0, 0, 0])                # checkpoint before any token: the old window
    st = s["state"].clone()
    old = st.clone()
    out, status = conv_ref.causal_conv1d(x, s["weight"], s["bias"], st, idx, cu, init, tidx, tlen)
    assert status == 0
    assert torch.equal(st[0], old[0])                   # padding slot never written
    assert torch.equal(st[2], old[2])                   # empty request: slot unchanged
    assert torch.equal(st[5], old[1])                   # checkpoint at 0 = request 0's old window
    # request 0 (3 tokens, window 4): one old row, then its 3 tokens
    assert torch.equal(st[1], torch.cat([old[1][3:], x[0:3]]))
    # request 3 starts fresh: zeros before its tokens, and its window is its last 4 tokens
    assert torch.equal(st[3], x[6:10])
    fresh = s["bias"] + s["weight"][:, 3] * x[4].float()
    assert torch.allclose(out[0][4].float(), (fresh / (1 + torch.exp(-fresh))).bfloat16().float())
    # request 4 (2 tokens) continues: last two old rows, then its tokens
    assert torch.equal(st[4], torch.cat([old[4][2:], x[10:12]]))


def test_oracle_rejects_bad_slots_without_writing():
    s = _small()
    x = torch.randn(5, s["C"], generator=s["g"]).bfloat16()
    st = s["state"].clone()
    old = st.clone()
    out, status = conv_ref.causal_conv1d(x, s["weight"], None, st, torch.tensor([9, 1]), torch.tensor([0, 2, 5]))
    assert status == conv_ref.BAD_SLOT
    assert torch.equal(out[0][:2], torch.zeros(2, s["C"], dtype=torch.bfloat16))
    assert torch.equal(st[[0, 2, 3, 4, 5]], old[[0, 2, 3, 4, 5]])
    out, status = conv_ref.causal_conv1d(x, s["weight"], None, st, torch.tensor([1, 2]), torch.tensor([0, 2, 5]),
                                         track_indices=torch.tensor([0, -3]), track_lens=torch.tensor([0, 1]))
    assert status == conv_ref.BAD_SLOT
    assert torch.equal(out[0][2:], torch.zeros(3, s["C"], dtype=torch.bfloat16))
