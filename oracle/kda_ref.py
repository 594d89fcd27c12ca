"""CPU restatement of the reference GLM KDA operator -- TEST INFRASTRUCTURE ONLY.

This module is the checker for the CUDA kernels in ``01-glm53-ascend_b200``.
Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
arm may import it, and only to compare against or to time as the CPU baseline.
The product path never calls it and has no CPU fallback.

Every function restates the reference's PyTorch oracle
(``bench/kda_chunk/kda_python.py``) in plain fp32 torch on the CPU, with the
fixes and extensions the B200 operator needs:

* ``recurrent`` follows ``kda_recur_torch`` (kda_python.py:190-309) but indexes
  the packed tensors with the packed position ``bos + t``. The reference reads
  ``[:, t]`` with the sequence-local ``t`` (kda_python.py:271-303), so every
  sequence after the first in a varlen batch reads the first sequence's tokens.
* ``chunk`` follows ``kda_chunk_torch`` (kda_python.py:41-188) and accepts
  sequence lengths that are not multiples of the chunk size: the last chunk of a
  sequence is zero-padded (k = v = q = 0, g = 0, beta = 0), which leaves the
  state and every real row unchanged.
* both take either the raw gate (``a``, ``b``, ``A_log``, ``dt_bias``,
  ``lower_bound``; kda_python.py:16-39) or the log-decay ``g`` and ``beta``
  directly (the prepared-gate form the benchmark configurations specify).
* ``prepared_recurrent`` restates the recurrence on host-prepared fp32 inputs
  (sgl-glm53-ascend-ops/csrc/kda/prepared_recurrent.cpp:610-713 and the Triton
  twin bench/_prepared_recurrent/bench_prepared_recurrent.py:62-127).
* ``move_intermediate_cache_kda`` restates the speculative-decoding commit the
  reference's MTP test runs after a verify (a gather of accepted checkpoints).

Parity is pinned against the reference's own code: ``tests/golden/make_golden.py``
runs ``kda_chunk_torch``, ``kda_recur_torch`` (one sequence per call, where it
is correct), the in-file ``_reference`` of ``tests/ops/test_kda_chunk.py`` and
the Triton ``_prepared_recurrent`` (interpreter mode) on seeded inputs and
commits their outputs; ``tests/test_oracle_golden.py`` checks this module
against those fixtures.

State pools are ``[slots, H, K, V]`` tensors with any strides (the production
pool is the K-contiguous view, stride(2) == 1). Slot 0 is the padding row: it
reads as a zero state and is never written (kda_python.py:105-108, 185-186).
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch

EPS = 1e-6


def _f32(x: torch.Tensor) -> torch.Tensor:
    return x.detach().to("cpu", torch.float32)


def _ints(x) -> list:
    if x is None:
        return None
    if isinstance(x, torch.Tensor):
        return [int(v) for v in x.detach().cpu().reshape(-1).tolist()]
    return [int(v) for v in x]


# ---------------------------------------------------------------------------
# Prologue: L2 norms, gate, beta (kda_python.py:16-39)
# ---------------------------------------------------------------------------

def prologue_raw(q, k, a, b, A_log, dt_bias, lower_bound: float, scale: float):
    """``kda_pre_torch`` (kda_python.py:16-39): qn, kn, g, beta in fp32.

    q, k, a: [1, T, H, K]; b: [1, T, H]; A_log: [H]; dt_bias: [H, K] or [H*K].
    """
    q, k, a, b = (_f32(t) for t in (q, k, a, b))
    H, K = k.shape[2], k.shape[3]
    qn = q / torch.sqrt((q * q).sum(-1, keepdim=True) + EPS) * scale
    kn = k / torch.sqrt((k * k).sum(-1, keepdim=True) + EPS)
    gate = _f32(A_log).reshape(H).exp()[None, None, :, None] * (
        a + _f32(dt_bias).reshape(H, K)[None, None])
    g = lower_bound * torch.sigmoid(gate)
    beta = torch.sigmoid(b)
    return qn, kn, g, beta


def prologue_log(q, k, g, beta, scale: float):
    """Same norms as ``prologue_raw``; the gate arrives as log-decay ``g``
    ([1, T, H, K] fp32) and ``beta`` ([1, T, H] fp32) directly."""
    q, k = _f32(q), _f32(k)
    qn = q / torch.sqrt((q * q).sum(-1, keepdim=True) + EPS) * scale
    kn = k / torch.sqrt((k * k).sum(-1, keepdim=True) + EPS)
    return qn, kn, _f32(g), _f32(beta)


# ---------------------------------------------------------------------------
# Token recurrence (kda_python.py:190-309, packed index fixed)
# ---------------------------------------------------------------------------

def recurrent(qn, kn, v, g, beta, pool: torch.Tensor, indices, cu_seqlens,
              intermediate: Optional[torch.Tensor] = None,
              track_indices=None, track_lens=None) -> torch.Tensor:
    """Token-at-a-time KDA over a varlen batch; returns fp32 output [1,T,H,V].

    ``pool`` ([slots,H,K,V], fp32, any strides) is updated in place: the final
    state of request i goes to ``indices[i]`` unless that is 0 or
    ``intermediate`` is given. ``intermediate`` ([reqs, steps, H, K, V]) gets
    the state after every step of request i at row i (the request's batch
    position, not its slot), skipped for slot 0 (kda_python.py:299-300).
    ``track_indices``/``track_lens``: request i's state after
    ``track_lens[i]`` of its own tokens goes to slot ``track_indices[i]``
    (0 = off; a length of 0 means the initial state; kda_python.py:264-294).
    """
    qn, kn, v, g, beta = (_f32(t) for t in (qn, kn, v, g, beta))
    T, H, K = kn.shape[1], kn.shape[2], kn.shape[3]
    V = v.shape[3]
    cu = _ints(cu_seqlens)
    slots = _ints(indices)
    tidx = _ints(track_indices)
    tlen = _ints(track_lens)
    decay = g.exp()
    out = torch.zeros(1, T, H, V, dtype=torch.float32)
    for seq in range(len(cu) - 1):
        bos, eos, slot = cu[seq], cu[seq + 1], slots[seq]
        if slot > 0:
            S = pool[slot].detach().to("cpu", torch.float32).clone()
        else:
            S = torch.zeros(H, K, V, dtype=torch.float32)
        ti = tidx[seq] if tidx is not None else 0
        tl = tlen[seq] if (tlen is not None and ti > 0) else -1
        if ti > 0 and tl == 0:
            pool[ti].copy_(S)
        for t in range(eos - bos):
            i = bos + t
            S = S * decay[0, i][:, :, None]
            pred = torch.einsum("hk,hkv->hv", kn[0, i], S)
            delta = (v[0, i] - pred) * beta[0, i][:, None]
            S = S + kn[0, i][:, :, None] * delta[:, None, :]
            if ti > 0 and t + 1 == tl:
                pool[ti].copy_(S)
            if intermediate is not None and slot > 0:
                intermediate[seq, t].copy_(S)
            out[0, i] = torch.einsum("hk,hkv->hv", qn[0, i], S)
        if intermediate is None and slot > 0:
            pool[slot].copy_(S)
    return out


# ---------------------------------------------------------------------------
# Chunked form (kda_python.py:41-188, ragged last chunk allowed)
# ---------------------------------------------------------------------------

def _chunk_tensors(qn, kn, v, g, beta, bos, eos, BT):
    """Slice one sequence and zero-pad it to whole chunks: [NT, BT, H, ...]."""
    n = eos - bos
    NT = (n + BT - 1) // BT
    pad = NT * BT - n

    def cut(x):
        x = x[0, bos:eos]
        if pad:
            x = torch.cat([x, x.new_zeros((pad,) + tuple(x.shape[1:]))], 0)
        return x.reshape((NT, BT) + tuple(x.shape[1:]))

    return NT, [cut(x) for x in (qn, kn, v, g, beta)]


def chunk(qn, kn, v, g, beta, pool: torch.Tensor, indices, cu_seqlens,
          track_indices=None, track_lens=None, BT: int = 64) -> torch.Tensor:
    """Chunk-BT WY/UT form of the same operator; returns fp32 [1,T,H,V].

    Per chunk (kda_python.py:127-182): gc = cumsum(g);
    A[r,c] = -beta_r sum_k k_r k_c e^{gc_r - gc_c} (c < r), solved by forward
    substitution into (I - A)^{-1} diag(beta); w = A (e^{gc} k), u = A v;
    v' = u - w S; o = (q e^{gc}) S + Aqk v' with Aqk[r,c] = sum_k q_r k_c
    e^{gc_r - gc_c} (c <= r); S = e^{gc_last} S + (k e^{gc_last - gc})^T v'.
    """
    qn, kn, v, g, beta = (_f32(t) for t in (qn, kn, v, g, beta))
    T, H, K = kn.shape[1], kn.shape[2], kn.shape[3]
    V = v.shape[3]
    cu = _ints(cu_seqlens)
    slots = _ints(indices)
    tidx = _ints(track_indices)
    tlen = _ints(track_lens)
    out = torch.zeros(1, T, H, V, dtype=torch.float32)
    strict = torch.tril(torch.ones(BT, BT, dtype=torch.bool), diagonal=-1)
    lower = torch.tril(torch.ones(BT, BT, dtype=torch.bool), diagonal=0)
    eye = torch.eye(BT, dtype=torch.float32)
    for seq in range(len(cu) - 1):
        bos, eos, slot = cu[seq], cu[seq + 1], slots[seq]
        if slot > 0:
            S = pool[slot].detach().to("cpu", torch.float32).clone()
        else:
            S = torch.zeros(H, K, V, dtype=torch.float32)
        ti = tidx[seq] if tidx is not None else 0
        tl = tlen[seq] if (tlen is not None and ti > 0) else -1
        if ti > 0 and tl == 0:
            pool[ti].copy_(S)
        if eos == bos:
            continue
        NT, (q_c, k_c, v_c, g_c, b_c) = _chunk_tensors(qn, kn, v, g, beta, bos, eos, BT)
        # [NT, H, BT, ...]
        q_c, k_c, v_c, g_c = (x.transpose(1, 2) for x in (q_c, k_c, v_c, g_c))
        b_c = b_c.transpose(1, 2)
        gc = g_c.cumsum(-2)
        o = torch.zeros_like(v_c)
        for c in range(NT):
            # Pairwise decayed products; every exponent on the kept triangle
            # is <= 0, as in kda_python.py:133-137 and :159-162.
            diff = gc[c][:, :, None, :] - gc[c][:, None, :, :]       # [H,r,c,K]
            dec = torch.where(lower[None, :, :, None], diff,
                              torch.full_like(diff, -float("inf"))).exp()
            Akk = torch.einsum("hrk,hck,hrck->hrc", k_c[c], k_c[c], dec)
            Aqk = torch.einsum("hrk,hck,hrck->hrc", q_c[c], k_c[c], dec)
            del dec, diff
            A = -(Akk * b_c[c][..., None]).masked_fill(~strict, 0.0)
            for i in range(1, BT):
                A[..., i, :i] = A[..., i, :i] + (A[..., i, :, None] * A[..., :, :i]).sum(-2)
            A = (A + eye) * b_c[c][..., None, :]
            w = A @ (gc[c].exp() * k_c[c])
            u = A @ v_c[c]
            Aqk = Aqk.masked_fill(~lower, 0.0)
            vnew = u - w @ S                                         # [H,BT,V]
            o[c] = (q_c[c] * gc[c].exp()) @ S + Aqk @ vnew
            if ti > 0 and c * BT < tl <= (c + 1) * BT:
                r = tl - c * BT
                gr = gc[c, :, r - 1]                                 # [H,K]
                Sr = S * gr.exp()[:, :, None]
                Sr = Sr + ((gr[:, None, :] - gc[c, :, :r]).exp() * k_c[c, :, :r]).transpose(1, 2) @ vnew[:, :r]
                pool[ti].copy_(Sr)
            gl = gc[c, :, -1]                                        # [H,K]
            S = S * gl.exp()[:, :, None]
            S = S + ((gl[:, None, :] - gc[c]).exp() * k_c[c]).transpose(1, 2) @ vnew
        n = eos - bos
        out[0, bos:eos] = o.transpose(1, 2).reshape(NT * BT, H, V)[:n]
        if slot > 0:
            pool[slot].copy_(S)
    return out


# ---------------------------------------------------------------------------
# Prepared-input recurrence (prepared_recurrent.cpp:610-713)
# ---------------------------------------------------------------------------

def prepared_recurrent(qn, kn, v, gdecay, beta, out, state, indices, starts,
                       track_indices=None, track_lens=None, track_state=False,
                       head_offset: int = 0, heads_per_launch: int = 4) -> None:
    """The recurrence on prepared fp32 inputs, heads [head_offset,
    head_offset + heads_per_launch), written into ``out`` (bf16, in place) and
    ``state`` (in place). qn/kn/gdecay: [..., T*H or T, H, D] fp32 with
    gdecay = exp(g); beta: [T*H] fp32; v/out: bf16. The Triton twin
    (bench_prepared_recurrent.py:62-127) walks one request; every request in
    ``indices`` is walked here.
    """
    H = state.shape[1]
    D = state.shape[2]
    qn, kn, gdecay = (_f32(t).reshape(-1, H, D) for t in (qn, kn, gdecay))
    vv = _f32(v).reshape(-1, H, D)
    bb = _f32(beta).reshape(-1, H)
    cu = _ints(starts)
    slots = _ints(indices)
    tidx = _ints(track_indices) if track_state else None
    tlen = _ints(track_lens) if track_state else None
    o = out.view(-1, H, D)
    heads = list(range(head_offset, min(H, head_offset + heads_per_launch)))
    for req in range(len(slots)):
        bos, eos, slot = cu[req], cu[req + 1], slots[req]
        for h in heads:
            S = state[slot, h].detach().to("cpu", torch.float32).clone() if slot > 0 \
                else torch.zeros(D, D, dtype=torch.float32)
            ti = tidx[req] if tidx is not None else 0
            tl = tlen[req] if ti > 0 else -1
            if ti > 0 and tl == 0:
                state[ti, h].copy_(S)
            for t in range(eos - bos):
                i = bos + t
                S = S * gdecay[i, h][:, None]
                pred = kn[i, h] @ S
                delta = (vv[i, h] - pred) * bb[i, h]
                S = S + kn[i, h][:, None] * delta[None, :]
                if ti > 0 and t + 1 == tl:
                    state[ti, h].copy_(S)
                o[i, h] = (qn[i, h] @ S).to(o.dtype)
            if slot > 0:
                state[slot, h].copy_(S)


# ---------------------------------------------------------------------------
# Speculative-decoding commit (move_intermediate_cache_kda)
# ---------------------------------------------------------------------------

def move_intermediate_cache_kda(dst, src, dst_indices, src_indices, step_indices,
                                h_block_size: int = 1) -> None:
    """The commit after a verify pass, as the reference's MTP test calls it
    (sgl-glm53-ascend-ops/tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:93-99):
    ``dst[:, dst_indices[i]] = src[:, src_indices[i], step_indices[i]]`` for
    every entry i, with dst ``[layers, slots, H, D, D]`` and src
    ``[layers, requests, steps, H, D, D]`` (any strides; elements are matched by
    logical index). The function itself (sgl_kernel_npu) is not in the
    reference tree; this restates the copy its call site implies. An entry with
    a negative step copies nothing; an index past its dimension raises.
    ``h_block_size`` is the original's heads-per-program tiling and does not
    change the result."""
    assert h_block_size >= 1
    for slot, req, step in zip(_ints(dst_indices), _ints(src_indices), _ints(step_indices)):
        if step < 0:
            continue
        if not (0 <= slot < dst.shape[1] and 0 <= req < src.shape[1] and step < src.shape[2]):
            raise IndexError(f"commit entry ({slot}, {req}, {step}) out of range")
        dst[:, slot].copy_(src[:, req, step])


# ---------------------------------------------------------------------------
# Whole-op mirrors of the torch ops (bf16 output, pool updated in place)
# ---------------------------------------------------------------------------

def kda_varlen_recurrent(*, A_log, a, dt_bias, q, k, v, b, initial_state_source,
                         initial_state_indices, cu_seqlens, lower_bound, scale,
                         intermediate_state=None, prefill=False,
                         track_state_indices=None, track_state_lens=None,
                         out_fp32: bool = False) -> torch.Tensor:
    """Oracle for ``sgl_glm53_ascend::kda_varlen_recurrent`` (raw gate).
    ``out_fp32`` returns the pre-cast fp32 output instead of the bf16 one."""
    qn, kn, g, beta = prologue_raw(q, k, a, b, A_log, dt_bias, lower_bound, scale)
    o = recurrent(qn, kn, v, g, beta, initial_state_source, initial_state_indices,
                  cu_seqlens, intermediate_state, track_state_indices, track_state_lens)
    return o if out_fp32 else o.to(torch.bfloat16)


def kda_varlen_chunk(*, A_log, a, dt_bias, q, k, v, b, initial_state_source,
                     initial_state_indices, cu_seqlens, lower_bound, scale,
                     prefill=False, track_state_indices=None,
                     track_state_lens=None, out_fp32: bool = False) -> torch.Tensor:
    """Oracle for ``sgl_glm53_ascend::kda_varlen_chunk`` (raw gate)."""
    qn, kn, g, beta = prologue_raw(q, k, a, b, A_log, dt_bias, lower_bound, scale)
    o = chunk(qn, kn, v, g, beta, initial_state_source, initial_state_indices,
              cu_seqlens, track_state_indices, track_state_lens)
    return o if out_fp32 else o.to(torch.bfloat16)


def kda_varlen_recurrent_g(*, q, k, v, g, beta, initial_state_source,
                           initial_state_indices, cu_seqlens, scale,
                           intermediate_state=None, prefill=False,
                           track_state_indices=None, track_state_lens=None,
                           out_fp32: bool = False) -> torch.Tensor:
    """Oracle for the log-gate recurrent op (g and beta given directly)."""
    qn, kn, g, beta = prologue_log(q, k, g, beta, scale)
    o = recurrent(qn, kn, v, g, beta, initial_state_source, initial_state_indices,
                  cu_seqlens, intermediate_state, track_state_indices, track_state_lens)
    return o if out_fp32 else o.to(torch.bfloat16)


def kda_varlen_chunk_g(*, q, k, v, g, beta, initial_state_source,
                       initial_state_indices, cu_seqlens, scale, prefill=False,
                       track_state_indices=None, track_state_lens=None,
                       out_fp32: bool = False) -> torch.Tensor:
    """Oracle for the log-gate chunk op (g and beta given directly)."""
    qn, kn, g, beta = prologue_log(q, k, g, beta, scale)
    o = chunk(qn, kn, v, g, beta, initial_state_source, initial_state_indices,
              cu_seqlens, track_state_indices, track_state_lens)
    return o if out_fp32 else o.to(torch.bfloat16)
