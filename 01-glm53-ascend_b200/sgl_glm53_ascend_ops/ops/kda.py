"""Keyword-only wrappers over ``torch.ops.sgl_glm53_ascend.*``.

Signatures are the reference's (``sgl_glm53_ascend_ops/ops/kda.py:6-235``) so
the sglang backend swaps this package in unchanged; ``kda_varlen_recurrent_g``
and ``kda_varlen_chunk_g`` are additions that take the fp32 log-decay ``g`` and
``beta`` directly instead of the raw gate (``a``, ``b``, ``A_log``,
``dt_bias``, ``lower_bound``).

All ops run asynchronously on the current CUDA stream, allocate only their
output (and, for the chunk op, a workspace from the caching allocator), never
copy metadata to the host, and may be captured in a CUDA graph.
"""

from typing import Optional

import torch


def prepared_recurrent(
    qn: torch.Tensor,
    kn: torch.Tensor,
    v: torch.Tensor,
    gdecay: torch.Tensor,
    beta: torch.Tensor,
    out: torch.Tensor,
    state: torch.Tensor,
    indices: torch.Tensor,
    starts: torch.Tensor,
    track_indices: Optional[torch.Tensor] = None,
    track_lens: Optional[torch.Tensor] = None,
    track_state: bool = False,
    head_offset: int = 0,
):
    """Recurrence on prepared fp32 ``qn``/``kn``/``gdecay`` (= exp(g))/``beta``
    for heads ``[head_offset, head_offset + 4)``; ``out`` and ``state`` are
    written in place (reference: ``prepared_recurrent.cpp:610-713``)."""
    return torch.ops.sgl_glm53_ascend.prepared_recurrent(
        qn, kn, v, gdecay, beta, out, state, indices, starts,
        track_indices, track_lens, track_state, head_offset,
    )


def kda_varlen_recurrent_v2(
    *,
    A_log: torch.Tensor,
    a: torch.Tensor,
    dt_bias: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    b: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    lower_bound: float,
    scale: float,
    intermediate_state: Optional[torch.Tensor] = None,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Registered under the v2 name the reference reserves for its next
    kernel; here it runs the same kernel as :func:`kda_varlen_recurrent`."""
    return torch.ops.sgl_glm53_ascend.kda_varlen_recurrent_v2(
        A_log=A_log, a=a, dt_bias=dt_bias, q=q, k=k, v=v, b=b,
        initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens,
        lower_bound=lower_bound, scale=scale, intermediate_state=intermediate_state,
        prefill=prefill, track_state_indices=track_state_indices,
        track_state_lens=track_state_lens,
    )


def kda_varlen_recurrent(
    *,
    A_log: torch.Tensor,
    a: torch.Tensor,
    dt_bias: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    b: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    lower_bound: float,
    scale: float,
    intermediate_state: Optional[torch.Tensor] = None,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Fused KDA varlen recurrence; returns the bf16 output, updates the state
    pool in place.

    Replaces the implementation-selection block inside sglang's
    ``glm_kda_varlen_recurrent_npu`` (reference ``ops/kda.py:92-115``). The
    caller's own validation runs first; the op checks what the kernels index
    against: dtypes, H == HV, K == V in {64, 128}, and the K-contiguous pool
    ([slots, H, K, V] with stride(2) == 1, stride(3) == K).

    Any head count, any number of requests and any lengths are served, in both
    regimes: decode/verify (``prefill=False``, at least one token per request,
    optional per-step ``intermediate_state`` checkpoints with no final state
    write) and token-recurrent prefill (``prefill=True``, optional prefix
    checkpoints via ``track_state_indices``/``track_state_lens``). Slot 0 is
    the padding row: zero initial state, never written.
    """
    return torch.ops.sgl_glm53_ascend.kda_varlen_recurrent(
        A_log=A_log, a=a, dt_bias=dt_bias, q=q, k=k, v=v, b=b,
        initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens,
        lower_bound=lower_bound, scale=scale, intermediate_state=intermediate_state,
        prefill=prefill, track_state_indices=track_state_indices,
        track_state_lens=track_state_lens,
    )


def kda_varlen_chunk_v2(
    *,
    A_log: torch.Tensor,
    a: torch.Tensor,
    dt_bias: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    b: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    lower_bound: float,
    scale: float,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """The v2 name of :func:`kda_varlen_chunk` (same kernel)."""
    return torch.ops.sgl_glm53_ascend.kda_varlen_chunk_v2(
        A_log=A_log, a=a, dt_bias=dt_bias, q=q, k=k, v=v, b=b,
        initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens,
        lower_bound=lower_bound, scale=scale, prefill=prefill,
        track_state_indices=track_state_indices, track_state_lens=track_state_lens,
    )


def kda_varlen_chunk(
    *,
    A_log: torch.Tensor,
    a: torch.Tensor,
    dt_bias: torch.Tensor,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    b: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    lower_bound: float,
    scale: float,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Chunked (64-token) KDA; returns the output, updates the state in place.

    The chunked form of :func:`kda_varlen_recurrent` (reference
    ``ops/kda.py:198-219``), minus ``intermediate_state``. Unlike the
    reference, sequence lengths need not be multiples of 64: a partial last
    chunk is masked in the kernel, so the op never reads ``cu_seqlens`` on the
    host. ``track_state_indices``/``track_state_lens``: slot
    ``track_state_indices[i]`` receives request i's state after
    ``track_state_lens[i]`` of its own tokens (0 = the initial state).
    """
    return torch.ops.sgl_glm53_ascend.kda_varlen_chunk(
        A_log=A_log, a=a, dt_bias=dt_bias, q=q, k=k, v=v, b=b,
        initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens,
        lower_bound=lower_bound, scale=scale, prefill=prefill,
        track_state_indices=track_state_indices, track_state_lens=track_state_lens,
    )


def kda_varlen_recurrent_g(
    *,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    scale: float,
    intermediate_state: Optional[torch.Tensor] = None,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """:func:`kda_varlen_recurrent` with the gate given as the fp32 log-decay
    ``g`` [1,T,H,K] and ``beta`` [1,T,H]; q and k are still L2-normalised in
    the kernel and q scaled by ``scale``."""
    return torch.ops.sgl_glm53_ascend.kda_varlen_recurrent_g(
        q=q, k=k, v=v, g=g, beta=beta, initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens, scale=scale,
        intermediate_state=intermediate_state, prefill=prefill,
        track_state_indices=track_state_indices, track_state_lens=track_state_lens,
    )


def kda_varlen_chunk_g(
    *,
    q: torch.Tensor,
    k: torch.Tensor,
    v: torch.Tensor,
    g: torch.Tensor,
    beta: torch.Tensor,
    initial_state_source: torch.Tensor,
    initial_state_indices: torch.Tensor,
    cu_seqlens: torch.Tensor,
    scale: float,
    prefill: bool = False,
    track_state_indices: Optional[torch.Tensor] = None,
    track_state_lens: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """:func:`kda_varlen_chunk` with the fp32 log-decay ``g`` and ``beta``."""
    return torch.ops.sgl_glm53_ascend.kda_varlen_chunk_g(
        q=q, k=k, v=v, g=g, beta=beta, initial_state_source=initial_state_source,
        initial_state_indices=initial_state_indices, cu_seqlens=cu_seqlens, scale=scale,
        prefill=prefill, track_state_indices=track_state_indices,
        track_state_lens=track_state_lens,
    )


def move_intermediate_cache_kda(
    dst: torch.Tensor,
    src: torch.Tensor,
    dst_indices: torch.Tensor,
    src_indices: torch.Tensor,
    step_indices: torch.Tensor,
    h_block_size: int = 1,
) -> None:
    """Speculative-decoding commit: ``dst[:, dst_indices[i]] =
    src[:, src_indices[i], step_indices[i]]`` in place, with ``dst`` the pool
    ``[layers, slots, H, D, D]`` and ``src`` the verify checkpoints
    ``[layers, requests, steps, H, D, D]``; a negative step copies nothing.
    Same positional call as sgl_kernel_npu's function of this name in the
    reference's MTP test (test_glm53_kda_mtp_state_view_ascendc.py:93-99)."""
    torch.ops.sgl_glm53_ascend.move_intermediate_cache_kda(
        dst, src, dst_indices, src_indices, step_indices, h_block_size)
