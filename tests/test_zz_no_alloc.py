"""The allocation-free chunk entry point, `kda_chunk_launch_no_alloc`.

Some hosts cannot give this library device memory: their own pools already
claim it, or they call in through a foreign-function layer that has no device
allocator. This entry point serves them by keeping the chunk prefill's only
scratch (the request order) in an array compiled into the library. The test
calls it through the C ABI twice in a row, with different batches, and checks
each result against `kda_chunk_launch` given a workspace, at the tolerances of
tests/kda_checks.py; it also checks the capacity limit. A third call uses a
batch of one long sequence over two heads, for which `kda_chunk_launch` with
a full workspace takes its split path while this entry point (no room for the
split path's records) always runs the fused kernel: the two paths must agree. The file name sorts
last so that a run stopping at the first failure has run everything else.
"""

import pytest
import torch

from kda_checks import assert_out_close, assert_state_close, clone_pool

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _batch(lengths, heads, seed):
    import kda_workloads as workloads
    w = workloads.config3(seed=seed, heads=heads, lengths=lengths)
    w.pool = (torch.randn(w.pool.shape[0], heads, 128, 128) * 0.1).transpose(-1, -2)
    return w.to(DEV)


def _args(abi, d, out, pool):
    return abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=pool, indices=d.indices,
                                 cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                 g=d.g, beta=d.beta)


def test_no_alloc_matches_workspace_entry_point_twice():
    from sgl_glm53_ascend_ops import abi

    for lengths, heads, seed in (([300, 64, 1, 129, 70], 4, 11), ([65, 200], 2, 12), ([2048], 2, 14)):
        d = _batch(lengths, heads, seed)
        pool_ref, pool_new = clone_pool(d.pool), clone_pool(d.pool)
        out_ref, out_new = torch.empty_like(d.v), torch.empty_like(d.v)
        nws = abi.chunk_workspace_bytes(d.indices.numel(), d.tokens, heads, 128)
        if lengths == [2048]:
            assert nws > 4096, "the workspace entry point should take its split path here"
        ws = torch.empty(max(nws, 1), dtype=torch.uint8, device=DEV)
        assert abi.chunk_launch(_args(abi, d, out_ref, pool_ref), ws, nws) == abi.KDA_OK
        assert abi.chunk_launch_no_alloc(_args(abi, d, out_new, pool_new)) == abi.KDA_OK
        torch.cuda.synchronize()
        assert_out_close(out_new.cpu(), out_ref.cpu())
        assert_state_close(pool_new.cpu(), pool_ref.cpu())


def test_no_alloc_rejects_batches_beyond_its_capacity():
    from sgl_glm53_ascend_ops import abi

    d = _batch([3, 4], 1, 13)
    args = _args(abi, d, torch.empty_like(d.v), clone_pool(d.pool))
    args.num_req = 1025                                   # one past KDA_CHUNK_STATIC_MAX_REQUESTS
    assert abi.chunk_launch_no_alloc(args) == 6           # KDA_ERR_TOO_LARGE, nothing launched
