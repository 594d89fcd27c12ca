"""Causal-conv front end of the KDA attention layer, and the layer's extend step.

sglang's attention backend (``AscendKDAAttnBackend.forward_extend``, exercised
by ``sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_prefix_ascendc.py:325-387``)
turns the layer's mixed q | k | v projection into the KDA op's inputs with a
depthwise causal conv1d (4 taps, SiLU) that keeps each request's last input
rows in a conv-state pool, then runs the KDA op. These functions run that
step on the B200 kernels: ``causal_conv1d`` and ``conv_qkv`` call the
``kda_causal_conv1d`` op (one pass over the projection, q, k and v written as
contiguous planes), ``kda_forward_extend`` chains it with ``kda_varlen_chunk``
(prefill) and ``kda_forward_decode`` with ``kda_varlen_recurrent`` (decode).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch


def causal_conv1d(
    x: torch.Tensor,
    weight: torch.Tensor,
    bias: Optional[torch.Tensor],
    conv_state: torch.Tensor,
    cache_indices: torch.Tensor,
    query_start_loc: torch.Tensor,
    has_initial_state: Optional[torch.Tensor] = None,
    track_conv_indices: Optional[torch.Tensor] = None,
    track_conv_lens: Optional[torch.Tensor] = None,
    activation: Optional[str] = "silu",
    num_parts: int = 1,
) -> torch.Tensor:
    """Depthwise causal conv1d over a varlen batch; updates ``conv_state`` in place.

    x [T, C] bf16 (channels contiguous), weight [C, W] (W <= 4), bias [C] or
    None, conv_state [slots, window, C] bf16 with W - 1 <= window <= 8 (the last
    ``window`` raw input rows of each slot's sequence, oldest first; slot 0
    is the padding row). A request continues from its slot's last W - 1 rows
    unless ``has_initial_state`` says otherwise, and afterwards its slot holds
    its last ``window`` rows. ``track_conv_indices[i] > 0`` stores the window
    ending after ``track_conv_lens[i]`` of request i's tokens in that slot.

    Returns [num_parts, T, C / num_parts] bf16 (with num_parts = 1: [T, C]).
    """
    if activation not in (None, "silu", "swish"):
        raise ValueError(f"causal_conv1d does not support activation {activation!r}")
    out = torch.ops.sgl_glm53_ascend.kda_causal_conv1d(
        x, weight, bias, conv_state, cache_indices, query_start_loc, has_initial_state,
        track_conv_indices, track_conv_lens, num_parts, activation is not None)
    return out[0] if num_parts == 1 else out


def conv_qkv(
    mixed: torch.Tensor,
    conv_weights: torch.Tensor,
    bias: Optional[torch.Tensor],
    conv_state: torch.Tensor,
    cache_indices: torch.Tensor,
    query_start_loc: torch.Tensor,
    head_dim: int = 128,
    has_initial_state: Optional[torch.Tensor] = None,
    track_conv_indices: Optional[torch.Tensor] = None,
    track_conv_lens: Optional[torch.Tensor] = None,
) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """The conv (SiLU) over the mixed q | k | v projection [T, 3 * H * head_dim],
    split into the [1, T, H, head_dim] q, k and v tensors the KDA ops take
    (each a contiguous plane of one output buffer)."""
    T, C = mixed.shape[-2], mixed.shape[-1]
    if C % (3 * head_dim) != 0:
        raise ValueError(f"mixed has {C} channels, not 3 x H x {head_dim}")
    H = C // (3 * head_dim)
    planes = torch.ops.sgl_glm53_ascend.kda_causal_conv1d(
        mixed.reshape(T, C) if mixed.dim() == 3 else mixed, conv_weights, bias, conv_state, cache_indices,
        query_start_loc, has_initial_state, track_conv_indices, track_conv_lens, 3, True)
    q, k, v = (planes[i].view(1, T, H, head_dim) for i in range(3))
    return q, k, v


def kda_forward_extend(
    *,
    mixed: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    conv_weights: torch.Tensor,
    conv_bias: Optional[torch.Tensor],
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    lower_bound: float,
    conv_state: torch.Tensor,
    temporal_state: torch.Tensor,
    cache_indices: torch.Tensor,
    query_start_loc: torch.Tensor,
    head_dim: int = 128,
    scale: Optional[float] = None,
    has_initial_state: Optional[torch.Tensor] = None,
    track_indices: Optional[torch.Tensor] = None,
    track_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One KDA layer's extend (prefill) step after its projections: the conv
    front end on ``mixed``, then the chunked KDA op with the raw gate.

    mixed [T, 3 * H * head_dim] bf16; a [1, T, H * head_dim] bf16 (gate input);
    b [1, T, H] bf16 (beta logits); conv_state [slots, window, C] bf16 and
    temporal_state [slots, H, K, V] fp32 (K-contiguous) share the slot
    numbering ``cache_indices``; ``track_indices``/``track_lens`` (slot and
    tokens of the request before the checkpoint) take the tracked-prefix
    checkpoint of both pools at the same position. A request that starts fresh
    (``has_initial_state`` false) reads zeros for the conv rows before its
    first token; its temporal slot is read as given (the caller clears the
    slot of a new request, as sglang does when it allocates one).
    Returns the KDA output [1, T, H, head_dim] bf16.
    """
    q, k, v = conv_qkv(mixed, conv_weights, conv_bias, conv_state, cache_indices, query_start_loc,
                       head_dim=head_dim, has_initial_state=has_initial_state,
                       track_conv_indices=track_indices, track_conv_lens=track_lens)
    T, H = q.shape[1], q.shape[2]
    return torch.ops.sgl_glm53_ascend.kda_varlen_chunk(
        A_log=A_log, a=a.reshape(1, T, H, head_dim), dt_bias=dt_bias, q=q, k=k, v=v,
        b=b.reshape(1, T, H), initial_state_source=temporal_state, initial_state_indices=cache_indices,
        cu_seqlens=query_start_loc, lower_bound=lower_bound,
        scale=head_dim ** -0.5 if scale is None else scale, prefill=True,
        track_state_indices=track_indices, track_state_lens=track_lens)


def kda_forward_decode(
    *,
    mixed: torch.Tensor,
    a: torch.Tensor,
    b: torch.Tensor,
    conv_weights: torch.Tensor,
    conv_bias: Optional[torch.Tensor],
    A_log: torch.Tensor,
    dt_bias: torch.Tensor,
    lower_bound: float,
    conv_state: torch.Tensor,
    temporal_state: torch.Tensor,
    cache_indices: torch.Tensor,
    query_start_loc: torch.Tensor,
    head_dim: int = 128,
    scale: Optional[float] = None,
    intermediate_state: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """One KDA layer's decode step after its projections: the conv front end
    on ``mixed`` (each request continues from its conv window), then the token
    recurrence with the raw gate. Same tensors as :func:`kda_forward_extend`;
    ``intermediate_state`` takes the recurrence's per-step checkpoints of a
    verify pass (its conv window then holds all of the step's draft tokens).
    Returns the KDA output [1, T, H, head_dim] bf16.
    """
    q, k, v = conv_qkv(mixed, conv_weights, conv_bias, conv_state, cache_indices, query_start_loc,
                       head_dim=head_dim)
    T, H = q.shape[1], q.shape[2]
    return torch.ops.sgl_glm53_ascend.kda_varlen_recurrent(
        A_log=A_log, a=a.reshape(1, T, H, head_dim), dt_bias=dt_bias, q=q, k=k, v=v,
        b=b.reshape(1, T, H), initial_state_source=temporal_state, initial_state_indices=cache_indices,
        cu_seqlens=query_start_loc, lower_bound=lower_bound,
        scale=head_dim ** -0.5 if scale is None else scale, intermediate_state=intermediate_state,
        prefill=False)
