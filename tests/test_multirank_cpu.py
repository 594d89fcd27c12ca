"""Multi-rank host logic on CPU (gloo, world size 2).

The operator shards by heads (tensor parallelism) or by requests (data
parallelism) with no exchange step. These tests run two gloo ranks that each
take their shard of a workload, compute it (with the CPU oracle standing in
for the kernel, which needs a GPU), and check that an all-gather of the head
shards reassembles the unsharded output and state exactly as a single rank
computes them; plus the max-over-ranks timing reduction the benchmark uses.
"""

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, result_path: str):
    sys.path[:0] = [str(ROOT), str(ROOT / "01-glm53-ascend_b200"), str(ROOT / "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import kda_ref
        from kda_workloads import Workload, config2

        torch.set_num_threads(1)
        w = config2(requests=6, heads=4, slots=9)
        shard = w.head_shard(rank, world)
        pool = shard.pool.transpose(-1, -2).clone().transpose(-1, -2)
        out = kda_ref.kda_varlen_recurrent_g(**dict(shard.kwargs(), initial_state_source=pool), out_fp32=True)
        outs = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(outs, out)
        pools = [torch.empty_like(pool.contiguous()) for _ in range(world)]
        dist.all_gather(pools, pool.contiguous())
        # max over ranks, as bench.py's Dist.max does with NCCL
        t = torch.tensor([float(rank + 1)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            torch.save({"out": torch.cat(outs, dim=2), "pool": torch.cat(pools, dim=1), "max": t.item()},
                       result_path)
    finally:
        dist.destroy_process_group()


def test_head_shards_reassemble_on_two_gloo_ranks(tmp_path):
    sys.path[:0] = [str(ROOT / "01-glm53-ascend_b200")]
    from oracle import kda_ref
    from kda_workloads import config2

    result = tmp_path / "r.pt"
    mp.start_processes(_worker, args=(2, _free_port(), str(result)), nprocs=2, start_method="spawn")
    got = torch.load(result)
    w = config2(requests=6, heads=4, slots=9)
    pool = w.pool.transpose(-1, -2).clone().transpose(-1, -2)
    ref = kda_ref.kda_varlen_recurrent_g(**dict(w.kwargs(), initial_state_source=pool), out_fp32=True)
    torch.testing.assert_close(got["out"], ref, rtol=1e-6, atol=1e-7)
    torch.testing.assert_close(got["pool"], pool.contiguous(), rtol=1e-6, atol=1e-7)
    assert got["max"] == 2.0


def _gather_worker(rank: int, world: int, port: int, result_path: str):
    sys.path[:0] = [str(ROOT), str(ROOT / "01-glm53-ascend_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import bench
        from kda_workloads import config5

        d = bench.Dist()
        d.world, d.rank, d.pg = world, rank, dist
        w = config5(heads=4, decode=3, prefills=1, prefill_len=5, slots=9)
        shard = w.head_shard(rank, world)
        got_q = d.gather_heads(shard.q, dim=2)                    # [1, T, H, D] along heads
        got_pool = d.gather_heads(shard.pool[1:3], dim=1)         # [slots, H, K, V] along heads
        if rank == 0:
            torch.save({"q": got_q, "pool": got_pool}, result_path)
    finally:
        dist.destroy_process_group()


def test_bench_gather_reassembles_head_shards(tmp_path):
    """bench.py's verification gather (Dist.gather_heads) puts every rank's
    head shard back in rank order, for token tensors and pool slices."""
    from kda_workloads import config5

    result = tmp_path / "g.pt"
    mp.start_processes(_gather_worker, args=(2, _free_port(), str(result)), nprocs=2, start_method="spawn")
    got = torch.load(result)
    w = config5(heads=4, decode=3, prefills=1, prefill_len=5, slots=9)
    assert torch.equal(got["q"], w.q)
    assert torch.equal(got["pool"], w.pool[1:3])


def test_head_shard_layout():
    sys.path[:0] = [str(ROOT / "01-glm53-ascend_b200")]
    from kda_workloads import config3

    w = config3(heads=8, lengths=[5, 3])
    s = w.head_shard(1, 4)
    assert s.q.shape[2] == 2 and s.pool.shape[1] == 2
    assert torch.equal(s.q, w.q[:, :, 2:4])
    assert s.pool.stride(2) == 1 and s.pool.stride(3) == 128     # K-contiguous, as the op requires
    with pytest.raises(AssertionError):
        w.head_shard(0, 3)
