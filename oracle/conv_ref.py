"""CPU restatement of the KDA layer's causal-conv front end -- TEST INFRASTRUCTURE ONLY.

This module is the checker for ``kda_conv_launch`` (``01-glm53-ascend_b200``,
``csrc/kda_conv.cu``). Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline arm may import it; the product path never calls it.

What it restates. The sglang attention backend that the reference plugs into
(``AscendKDAAttnBackend.forward_extend``, exercised by
``sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387``)
runs a depthwise causal conv1d over the "mixed" q|k|v projection of each
sequence before the KDA op, keeping each request's last input rows in a conv
state pool ``[slots, window, channels]`` (time-major, channels contiguous;
``window`` is 3 or 6 rows there for a 4-tap kernel). sglang's own conv code is
not in the reference tree or in this image, so the arithmetic follows the
published causal-conv1d algorithm (Dao-AILab ``causal_conv1d_fn`` semantics,
as restated in vLLM 0.22's CPU ``causal_conv1d_torch``):

    out[t, c] = act(bias[c] + sum_{k<W} weight[c, k] * xin[t + k, c])

over ``xin`` = the W-1 rows before the sequence (from the state when the
request continues, zeros otherwise) followed by the sequence's rows, with
SiLU as the activation. The state rules are the ones the reference test
asserts:

* a request that continues reads the LAST W-1 rows of its slot
  (``conv[0][source, -3:]`` compared at ``:373`` and ``:383``);
* after the call the slot holds the last ``window`` rows of
  (old window ++ the request's rows): a sliding window of raw inputs
  (``:372-373``, ``:383``); a request that does not continue starts from zeros;
* the tracked-prefix checkpoint slot receives the ``window`` raw rows ending at
  the tracked position (``track_conv_indices = arange(cut - window, cut)``,
  ``:353`` and ``:372``), rows before the sequence coming from the old window;
* slot 0 is the padding row (as in the KDA state pool): it reads as zeros and
  is never written; every other slot is untouched (``:384-386``).

Parity is pinned against vLLM 0.22's ``causal_conv1d_torch`` by
``tests/golden/make_conv_golden.py`` (fixtures under ``tests/golden/``).

Arithmetic: fp32, taps summed in order k = 0..W-1 after the bias, SiLU as
``a / (1 + exp(-a))``, one rounding to bf16 at the end.
"""

from __future__ import annotations

from typing import Optional

import torch

# Device status codes (include/kda_b200.h).
BAD_SLOT = 0x102
BAD_SEQLENS = 0x103


def _silu(a: torch.Tensor) -> torch.Tensor:
    return a / (1.0 + torch.exp(-a))


def causal_conv1d(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor],
                  conv_state: torch.Tensor, cache_indices: torch.Tensor, cu_seqlens: torch.Tensor,
                  has_initial_state: Optional[torch.Tensor] = None,
                  track_indices: Optional[torch.Tensor] = None,
                  track_lens: Optional[torch.Tensor] = None,
                  activation: Optional[str] = "silu", num_parts: int = 1,
                  out_fp32: bool = False):
    """Conv front end over a varlen batch; updates ``conv_state`` in place.

    x [T, C] (bf16 or fp32), weight [C, W], bias [C] or None,
    conv_state [slots, window, C] (bf16), cache_indices [R], cu_seqlens [R+1],
    has_initial_state [R] bool or None (None: every request continues from its
    slot), track_indices / track_lens [R] or None (checkpoint slot, 0 = none;
    tokens of the request before the checkpoint).

    Returns ``(out, status)``: out [num_parts, T, C / num_parts] (bf16, or the
    fp32 pre-cast values with ``out_fp32``), every token row written (zeros for
    tokens no request covers and for rejected requests); status the first
    device error code the kernel would report (0 if none).
    """
    T, C = x.shape
    W = weight.shape[1]
    slots, window = conv_state.shape[0], conv_state.shape[1]
    assert window >= W - 1 and C % num_parts == 0
    xf = x.float()
    wf = weight.float()
    bf = bias.float() if bias is not None else None
    y = torch.zeros(T, C, dtype=torch.float32)
    old = conv_state.clone()
    status = 0
    R = cache_indices.numel()
    for r in range(R):
        bos, eos = int(cu_seqlens[r]), int(cu_seqlens[r + 1])
        slot = int(cache_indices[r])
        if bos < 0 or eos < bos or eos > T:
            status = status or BAD_SEQLENS
            continue
        if not 0 <= slot < slots:
            status = status or BAD_SLOT
            continue
        tslot = int(track_indices[r]) if track_indices is not None else 0
        if not 0 <= tslot < slots:
            status = status or BAD_SLOT
            continue
        init = slot > 0 and (has_initial_state is None or bool(has_initial_state[r]))
        prev = old[slot].float() if init else torch.zeros(window, C)
        hist = torch.cat([prev, xf[bos:eos]], 0)                 # [window + len, C]
        xin = hist[window - (W - 1):]                             # [W - 1 + len, C]
        n = eos - bos
        acc = bf.expand(n, C).clone() if bf is not None else torch.zeros(n, C)
        for k in range(W):
            acc = acc + wf[:, k] * xin[k:k + n]
        y[bos:eos] = _silu(acc) if activation in ("silu", "swish") else acc
        if tslot > 0:
            tlen = int(track_lens[r])
            if 0 <= tlen <= n:
                conv_state[tslot] = hist[tlen:tlen + window].to(conv_state.dtype)
        if slot > 0 and n > 0:
            conv_state[slot] = hist[n:n + window].to(conv_state.dtype)
    out = y if out_fp32 else y.to(torch.bfloat16)
    Cp = C // num_parts
    return out.view(T, num_parts, Cp).transpose(0, 1).contiguous(), status
