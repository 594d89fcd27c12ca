"""Pin ``oracle/kda_ref.py`` to the reference's own outputs (CPU only).

The fixtures under ``tests/golden/`` were produced by the reference's code
(``kda_recur_torch``/``kda_chunk_torch`` of bench/kda_chunk/kda_python.py, the
in-file ``_reference`` of tests/ops/test_kda_chunk.py, and the Triton
``_prepared_recurrent`` of bench/_prepared_recurrent/bench_prepared_recurrent.py
run by the Triton interpreter); ``tests/golden/make_golden.py`` regenerates them.

Both sides are fp32 on identical inputs with a different summation order, so
fp32 outputs and states agree to ~1e-6. Outputs the reference returns in bf16
may differ by one bf16 ulp where the fp32 value sits on a rounding boundary.
"""

import numpy as np
import pytest
import torch

from golden_io import bf16, expected_pool, kcontig, load, raw_kwargs
from oracle import kda_ref

# fp32 vs fp32, different summation order.
F32_RTOL, F32_ATOL = 1e-4, 1e-6
# bf16 vs bf16: one ulp (2^-8 relative) on boundary cases.
BF16_RTOL, BF16_ATOL = 8e-3, 1e-6
# The reference's own chunk-vs-recurrence bar (test_kda_chunk.py:55-56).
CHUNK_RTOL, CHUNK_ATOL = 2e-3, 1e-4


def _check_pool(pool, f, rtol=F32_RTOL, atol=F32_ATOL):
    torch.testing.assert_close(pool.float(), expected_pool(f), rtol=rtol, atol=atol)


def test_cfg1_recurrent_loggate():
    """BASELINE config 1, two sequences, via the fixed packed indexing."""
    f = load("cfg1_recurrent_loggate")
    pool = kcontig(f["pool_in"])
    out = kda_ref.kda_varlen_recurrent_g(
        q=bf16(f["q"]), k=bf16(f["k"]), v=bf16(f["v"]).float(),
        g=torch.from_numpy(f["g"]), beta=torch.from_numpy(f["beta"]),
        initial_state_source=pool, initial_state_indices=torch.from_numpy(f["indices"]),
        cu_seqlens=torch.from_numpy(f["cu_seqlens"]), scale=float(f["scale"]), out_fp32=True)
    torch.testing.assert_close(out, torch.from_numpy(f["out"]), rtol=F32_RTOL, atol=F32_ATOL)
    _check_pool(pool, f)


@pytest.mark.parametrize("name", ["recur_raw_tracked_d64", "recur_raw_tracked_d128",
                                  "recur_raw_varlen"])
def test_recurrent_raw(name):
    f = load(name)
    pool = kcontig(f["pool_in"])
    out = kda_ref.kda_varlen_recurrent(**raw_kwargs(f), initial_state_source=pool)
    torch.testing.assert_close(out.float(), torch.from_numpy(f["out"]),
                               rtol=BF16_RTOL, atol=BF16_ATOL)
    _check_pool(pool, f)


def test_recurrent_intermediate_checkpoints():
    """Per-step checkpoints by batch row; slot 0 request writes none; no final write."""
    f = load("recur_raw_intermediate")
    pool = kcontig(f["pool_in"])
    D = pool.shape[-1]
    H = pool.shape[1]
    noise = torch.randn(3, 4, H, D, D).transpose(-1, -2)
    mid = noise.transpose(-1, -2).clone().transpose(-1, -2)
    out = kda_ref.kda_varlen_recurrent(**raw_kwargs(f), initial_state_source=pool,
                                       intermediate_state=mid)
    torch.testing.assert_close(out.float(), torch.from_numpy(f["out"]),
                               rtol=BF16_RTOL, atol=BF16_ATOL)
    rows = f["mid_out_rows"].tolist()
    torch.testing.assert_close(mid[rows], torch.from_numpy(f["mid_out"]),
                               rtol=F32_RTOL, atol=F32_ATOL)
    # Row 1 (slot 0) is never written, and the pool keeps its pre-verify values.
    assert torch.equal(mid[1], noise[1])
    assert torch.equal(pool, kcontig(f["pool_in"]))
    assert f["pool_out_slots"].size == 0


CHUNK_FIXTURES = ["chunk_raw_tracked", "chunktest_ragged_varlen", "chunktest_zero_slot",
                  "chunktest_track_at_0", "chunktest_track_mid_chunk",
                  "chunktest_track_at_end"]


@pytest.mark.parametrize("name", CHUNK_FIXTURES)
def test_chunk_matches_reference_chunk(name):
    f = load(name)
    pool = kcontig(f["pool_in"])
    out = kda_ref.kda_varlen_chunk(**raw_kwargs(f), initial_state_source=pool)
    ref = torch.from_numpy(f["out"])
    if name.startswith("chunktest"):
        # The chunk test's _reference returns fp32; compare before the cast.
        qn, kn, g, beta = kda_ref.prologue_raw(
            bf16(f["q"]), bf16(f["k"]), bf16(f["a"]), bf16(f["b"]),
            torch.from_numpy(f["A_log"]), torch.from_numpy(f["dt_bias"]),
            float(f["lower_bound"]), float(f["scale"]))
        pool2 = kcontig(f["pool_in"])
        kw = raw_kwargs(f)
        o32 = kda_ref.chunk(qn, kn, bf16(f["v"]), g, beta, pool2, kw["initial_state_indices"],
                            kw["cu_seqlens"], kw.get("track_state_indices"),
                            kw.get("track_state_lens"))
        torch.testing.assert_close(o32, ref, rtol=1e-3, atol=1e-6)
    else:
        torch.testing.assert_close(out.float(), ref, rtol=BF16_RTOL, atol=BF16_ATOL)
    _check_pool(pool, f, rtol=1e-3, atol=1e-6)


@pytest.mark.parametrize("name", CHUNK_FIXTURES)
def test_recurrence_matches_reference_chunk(name):
    """The token recurrence reproduces the chunked reference at its own bar."""
    f = load(name)
    pool = kcontig(f["pool_in"])
    out = kda_ref.kda_varlen_recurrent(**raw_kwargs(f), initial_state_source=pool,
                                       prefill=True)
    torch.testing.assert_close(out.float(), torch.from_numpy(f["out"]),
                               rtol=CHUNK_RTOL, atol=CHUNK_ATOL)
    _check_pool(pool, f, rtol=CHUNK_RTOL, atol=CHUNK_ATOL)


def test_prepared_matches_triton():
    f = load("prepared_triton")
    state = torch.from_numpy(f["state_in"]).clone()
    out = torch.zeros(bf16(f["out"]).shape, dtype=torch.bfloat16)
    kda_ref.prepared_recurrent(
        torch.from_numpy(f["qn"]), torch.from_numpy(f["kn"]), bf16(f["v"]),
        torch.from_numpy(f["gdecay"]), torch.from_numpy(f["beta"]), out, state,
        torch.from_numpy(f["indices"]), torch.from_numpy(f["starts"]),
        torch.from_numpy(f["track_indices"]), torch.from_numpy(f["track_lens"]),
        track_state=True, head_offset=0)
    torch.testing.assert_close(out.float(), bf16(f["out"]).float(), rtol=BF16_RTOL,
                               atol=1e-6)
    torch.testing.assert_close(state, torch.from_numpy(f["state_out"]), rtol=F32_RTOL,
                               atol=F32_ATOL)


def test_ragged_chunk_equals_recurrence():
    """Lengths that are not multiples of 64 in the chunk form."""
    torch.manual_seed(4)
    H, D = 2, 64
    cu = torch.tensor([0, 37, 37, 170, 171])
    T = int(cu[-1])
    q, k, v = (torch.randn(1, T, H, D).bfloat16() for _ in range(3))
    g = torch.nn.functional.logsigmoid(torch.randn(1, T, H, D)).clamp(-5, 0)
    beta = torch.sigmoid(torch.randn(1, T, H))
    pool_a = (torch.randn(6, H, D, D) * 0.1).transpose(-1, -2)
    pool_b = pool_a.transpose(-1, -2).clone().transpose(-1, -2)
    idx = torch.tensor([1, 0, 3, 5])
    kw = dict(q=q, k=k, v=v, g=g, beta=beta, initial_state_indices=idx, cu_seqlens=cu,
              scale=D ** -0.5, out_fp32=True, track_state_indices=torch.tensor([2, 0, 4, 0]),
              track_state_lens=torch.tensor([20, 0, 100, 0]))
    oa = kda_ref.kda_varlen_recurrent_g(initial_state_source=pool_a, **kw)
    ob = kda_ref.kda_varlen_chunk_g(initial_state_source=pool_b, **kw)
    torch.testing.assert_close(ob, oa, rtol=1e-4, atol=1e-6)
    torch.testing.assert_close(pool_b, pool_a, rtol=1e-4, atol=1e-6)
