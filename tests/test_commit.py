"""The speculative-decoding commit, ``move_intermediate_cache_kda``.

The reference's MTP regression (tests/integration/test_glm53_kda_mtp_state_view_ascendc.py:77-116)
runs a 4-token verify that writes per-step checkpoints, commits the accepted
step into the pool with sgl_kernel_npu's ``move_intermediate_cache_kda``, and
demands that the committed pool equal, bit for bit, the pool a plain decode of
the same tokens leaves behind. The same flow is checked here on the CPU oracle
(which pins the oracle's commit to the reference test's own assertion) and on
the GPU through the B200 ops; the GPU kernel is also compared with the oracle
on gathers with every stride pattern, negative steps, int64 indices and an
out-of-range index (reported through the status word, nothing written).
"""

import pytest
import torch

from oracle import kda_ref

DEV = "cuda"
H, D = 4, 128


def _inputs(tokens, seed):
    g = torch.Generator().manual_seed(seed)
    q, k, v, a = ((torch.randn(1, tokens, H, D, generator=g)).bfloat16() for _ in range(4))
    b = torch.randn(1, tokens, H, generator=g).bfloat16()
    return dict(q=q, k=k, v=v, a=a, b=b, cu_seqlens=torch.tensor([0, tokens], dtype=torch.int32))


def _layer(seed=17):
    g = torch.Generator().manual_seed(seed)
    return dict(A_log=torch.randn(H, generator=g), dt_bias=torch.randn(H, D, generator=g), lower_bound=-10.0,
                scale=D ** -0.5)


def _pool():
    # Two slots (0 = padding, 1 = the request), K-contiguous as the ops require.
    return torch.zeros(2, H, D, D).transpose(-1, -2)


def _mtp_flow(run, commit, to_dev=lambda t: t):
    """Prefill 26 tokens, then verify 4 with checkpoints and commit step 3;
    returns (plain pool, committed pool, plain verify out, checkpointed out)."""
    layer = {n: to_dev(t) if isinstance(t, torch.Tensor) else t for n, t in _layer().items()}
    indices = to_dev(torch.tensor([1], dtype=torch.int32))
    baseline, speculative = to_dev(_pool()), to_dev(_pool())
    pre = {n: to_dev(t) for n, t in _inputs(26, 1).items()}
    run(baseline, pre, indices, layer, prefill=True)
    run(speculative, pre, indices, layer, prefill=True)
    ver = {n: to_dev(t) for n, t in _inputs(4, 2).items()}
    ref = run(baseline, ver, indices, layer, prefill=False)
    scratch = to_dev(torch.zeros(1, 1, 4, H, D, D).transpose(-1, -2))   # [layers, req, steps, H, K, V]
    got = run(speculative, ver, indices, layer, prefill=False, intermediate=scratch[0])
    # Both sides through their physical [V][K] views (the reference test commits into
    # the destination's physical view for the same reason).
    commit(speculative.unsqueeze(0).transpose(-1, -2), scratch.transpose(-1, -2),
           to_dev(torch.tensor([1], dtype=torch.int32)), to_dev(torch.tensor([0], dtype=torch.int32)),
           to_dev(torch.tensor([3], dtype=torch.int32)))
    return baseline, speculative, ref, got


def test_oracle_commit_reproduces_plain_decode():
    def run(pool, x, indices, layer, prefill, intermediate=None):
        return kda_ref.kda_varlen_recurrent(**x, **layer, initial_state_source=pool, initial_state_indices=indices,
                                            intermediate_state=intermediate, prefill=prefill)

    baseline, speculative, ref, got = _mtp_flow(run, kda_ref.move_intermediate_cache_kda)
    assert torch.equal(ref, got)
    assert torch.equal(baseline, speculative)
    assert speculative.abs().sum() > 0


def test_oracle_commit_semantics():
    dst = torch.zeros(2, 5, 3, 4, 4)
    src = torch.randn(2, 3, 6, 3, 4, 4)
    kda_ref.move_intermediate_cache_kda(dst, src, torch.tensor([4, 1, 2]), torch.tensor([0, 2, 1]),
                                        torch.tensor([5, -1, 0]))
    assert torch.equal(dst[:, 4], src[:, 0, 5]) and torch.equal(dst[:, 2], src[:, 1, 0])
    assert not dst[:, 1].any() and not dst[:, 0].any() and not dst[:, 3].any()
    with pytest.raises(IndexError):
        kda_ref.move_intermediate_cache_kda(dst, src, torch.tensor([5]), torch.tensor([0]), torch.tensor([0]))


# ---------------------------------------------------------------------------
# GPU: the B200 ops
# ---------------------------------------------------------------------------

@pytest.fixture(scope="module")
def ops():
    from sgl_glm53_ascend_ops import ops as _ops
    return _ops


@pytest.mark.gpu
def test_gpu_commit_reproduces_plain_decode(ops):
    def run(pool, x, indices, layer, prefill, intermediate=None):
        return ops.kda_varlen_recurrent(**x, **layer, initial_state_source=pool, initial_state_indices=indices,
                                        intermediate_state=intermediate, prefill=prefill)

    baseline, speculative, ref, got = _mtp_flow(run, ops.move_intermediate_cache_kda, lambda t: t.to(DEV))
    torch.cuda.synchronize()
    assert torch.equal(ref, got), "verify output differs from the plain decode"
    assert torch.equal(baseline, speculative), "committed state differs from the plain decode"
    assert speculative.abs().sum() > 0


def _gather_case(seed, dst_t, src_t, Dm=128, index_dtype=torch.int32):
    g = torch.Generator().manual_seed(seed)
    L, slots, R, steps, Hh = 2, 7, 3, 4, 3
    dst = torch.randn(L, slots, Hh, Dm, Dm, generator=g)
    src = torch.randn(L, R, steps, Hh, Dm, Dm, generator=g)
    dst = dst.transpose(-1, -2).contiguous().transpose(-1, -2) if dst_t else dst
    src = src.transpose(-1, -2).contiguous().transpose(-1, -2) if src_t else src
    idx = [torch.tensor(x, dtype=index_dtype) for x in ([5, 2, 6, 1], [0, 2, 1, 2], [3, -1, 0, 2])]
    return dst, src, idx


@pytest.mark.gpu
@pytest.mark.parametrize("dst_t,src_t", [(False, False), (True, True), (True, False), (False, True)])
@pytest.mark.parametrize("Dm", (64, 128))
def test_gpu_commit_matches_oracle(ops, dst_t, src_t, Dm):
    dst, src, idx = _gather_case(3, dst_t, src_t, Dm)
    before = dst.clone()
    ddst = dst.transpose(-1, -2).to(DEV).transpose(-1, -2) if dst_t else dst.to(DEV)
    dsrc = src.transpose(-1, -2).to(DEV).transpose(-1, -2) if src_t else src.to(DEV)
    assert ddst.stride() == dst.stride() and dsrc.stride() == src.stride()
    ops.move_intermediate_cache_kda(ddst, dsrc, *[i.to(DEV) for i in idx])
    kda_ref.move_intermediate_cache_kda(dst, src, *idx)
    torch.cuda.synchronize()
    assert torch.equal(ddst.cpu(), dst)
    assert torch.equal(dst[:, 2], before[:, 2]), "a negative step must copy nothing"


@pytest.mark.gpu
def test_gpu_commit_int64_indices_and_abi(ops):
    from sgl_glm53_ascend_ops import abi
    dst, src, idx = _gather_case(4, True, True)
    a, b = dst.transpose(-1, -2).to(DEV).transpose(-1, -2), dst.transpose(-1, -2).to(DEV).transpose(-1, -2)
    dsrc = src.transpose(-1, -2).to(DEV).transpose(-1, -2)
    ops.move_intermediate_cache_kda(a, dsrc, *[i.to(DEV) for i in idx])
    i64 = [i.long().to(DEV) for i in idx]
    assert abi.commit_launch(abi.commit_args_from_tensors(b, dsrc, *i64)) == abi.KDA_OK
    torch.cuda.synchronize()
    assert torch.equal(a, b)


@pytest.mark.gpu
def test_gpu_commit_bad_index_reports_and_skips(ops):
    from sgl_glm53_ascend_ops import abi
    dst, src, _ = _gather_case(5, True, True)
    ddst = dst.transpose(-1, -2).to(DEV).transpose(-1, -2)
    dsrc = src.transpose(-1, -2).to(DEV).transpose(-1, -2)
    status = torch.zeros(1, dtype=torch.int32, device=DEV)
    idx = [torch.tensor(x, dtype=torch.int32, device=DEV) for x in ([7, 1], [0, 0], [0, 4])]   # slot 7, step 4: out of range
    assert abi.commit_launch(abi.commit_args_from_tensors(ddst, dsrc, *idx, status=status)) == abi.KDA_OK
    torch.cuda.synchronize()
    assert status.item() == 0x102
    assert torch.equal(ddst.cpu(), dst), "an out-of-range entry must not write"


@pytest.mark.gpu
def test_gpu_commit_rejections(ops):
    dst = torch.zeros(1, 3, 2, 64, 64, device=DEV)
    src = torch.zeros(1, 2, 2, 2, 64, 64, device=DEV)
    i = torch.zeros(1, dtype=torch.int32, device=DEV)
    with pytest.raises(RuntimeError, match="same length"):
        ops.move_intermediate_cache_kda(dst, src, i, i, torch.zeros(2, dtype=torch.int32, device=DEV))
    with pytest.raises(RuntimeError, match="D x D blocks"):
        ops.move_intermediate_cache_kda(dst, torch.zeros(1, 2, 2, 2, 32, 32, device=DEV), i, i, i)
