"""Seeded synthetic inputs with the shapes and value distributions of the
benchmark configurations (the reference publishes no dataset for this path).

Test and benchmark infrastructure, not part of the operator package: it
imports only torch, so the benchmark's CPU reference arm can use it without
loading any library of this repository.

Every tensor is drawn on the CPU with ``torch.manual_seed`` so a workload is
the same on any machine, then moved to ``device``:

* q, k, v ~ N(0, 1) in bf16;
* g = clamp(logsigmoid(N(0, 1)), -5, 0) per (token, head, key channel), fp32;
* beta = sigmoid(N(0, 1)) per (token, head), fp32;
* state pool ~ 0.1 N(0, 1), fp32, allocated [slots, H, V, K] and viewed as the
  K-contiguous [slots, H, K, V] pool the op requires; slot 0 is the padding
  row and starts at zero.

Configurations (BASELINE.json ``configs``):
  1: two sequences [0, 37, 128], H=4, D=64
  2: decode, 256 requests x 1 token, H=32, D=128, pool of 512 slots,
     indices = randperm(511)[:256] + 1
  3: varlen prefill, lengths randint(512, 8193, (8,)) from seed 1, H=32, D=128,
     zero initial state in slots 1..8
  4: one sequence of 131072 tokens, H=32 (sharded by heads), D=128
  5: mixed batch, 64 decode requests + 4 x 2048-token prefills, pool of 1024

plus ``conv_frontend``: the causal-conv front end's inputs for a batch of
request lengths (the mixed q | k | v projection ~ 0.2 N(0, 1) bf16, 4-tap
weights ~ 0.1 N(0, 1) fp32, a bf16 conv-state pool ~ 0.1 N(0, 1); requests
in slots 1..R), the shapes of the reference's backend test at any H.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import torch


@dataclass
class Workload:
    name: str
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    g: torch.Tensor
    beta: torch.Tensor
    pool: torch.Tensor
    indices: torch.Tensor
    cu_seqlens: torch.Tensor
    scale: float
    lengths: list = field(default_factory=list)

    @property
    def tokens(self) -> int:
        return self.q.shape[1]

    @property
    def heads(self) -> int:
        return self.q.shape[2]

    @property
    def dim(self) -> int:
        return self.q.shape[3]

    def to(self, device) -> "Workload":
        def mv(t):
            return t.to(device)

        pool = self.pool.transpose(-1, -2).to(device).transpose(-1, -2)
        return Workload(self.name, mv(self.q), mv(self.k), mv(self.v), mv(self.g), mv(self.beta), pool,
                        mv(self.indices), mv(self.cu_seqlens), self.scale, list(self.lengths))

    def kwargs(self) -> dict:
        """Keyword arguments of the log-gate ops."""
        return dict(q=self.q, k=self.k, v=self.v, g=self.g, beta=self.beta,
                    initial_state_source=self.pool, initial_state_indices=self.indices,
                    cu_seqlens=self.cu_seqlens, scale=self.scale)

    def head_shard(self, rank: int, world: int) -> "Workload":
        """Heads [rank*H/world, (rank+1)*H/world) with their slice of the pool:
        the layout tensor parallelism by heads gives each GPU. No data moves
        between ranks; each shard is a complete, independent problem."""
        H = self.heads
        assert H % world == 0, f"{H} heads do not split over {world} ranks"
        lo, hi = rank * H // world, (rank + 1) * H // world
        pool = self.pool[:, lo:hi].transpose(-1, -2).contiguous().transpose(-1, -2)
        return Workload(f"{self.name}[h{lo}:{hi}]", self.q[:, :, lo:hi].contiguous(),
                        self.k[:, :, lo:hi].contiguous(), self.v[:, :, lo:hi].contiguous(),
                        self.g[:, :, lo:hi].contiguous(), self.beta[:, :, lo:hi].contiguous(), pool,
                        self.indices, self.cu_seqlens, self.scale, list(self.lengths))


def _pool(slots: int, H: int, D: int, zero_slots=(0,)) -> torch.Tensor:
    pool = (torch.randn(slots, H, D, D) * 0.1).transpose(-1, -2)
    for s in zero_slots:
        pool[s] = 0
    return pool


def _tokens(T: int, H: int, D: int):
    q, k, v = (torch.randn(1, T, H, D).bfloat16() for _ in range(3))
    g = torch.nn.functional.logsigmoid(torch.randn(1, T, H, D)).clamp(-5.0, 0.0)
    beta = torch.sigmoid(torch.randn(1, T, H))
    return q, k, v, g, beta


def _cu(lengths) -> torch.Tensor:
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + int(n))
    return torch.tensor(cu, dtype=torch.int32)


def config1(seed: int = 0) -> Workload:
    torch.manual_seed(seed)
    H, D = 4, 64
    lengths = [37, 91]
    q, k, v, g, beta = _tokens(128, H, D)
    pool = _pool(3, H, D)
    return Workload("cfg1", q, k, v, g, beta, pool, torch.tensor([1, 2], dtype=torch.int32),
                    _cu(lengths), D ** -0.5, lengths)


def config2(seed: int = 0, requests: int = 256, heads: int = 32, slots: int = 512,
            pool_scale: float = 0.1) -> Workload:
    torch.manual_seed(seed)
    D = 128
    q, k, v, g, beta = _tokens(requests, heads, D)
    pool = _pool(slots, heads, D)
    indices = (torch.randperm(slots - 1)[:requests] + 1).to(torch.int32)
    return Workload("cfg2", q, k, v, g, beta, pool, indices, _cu([1] * requests), D ** -0.5,
                    [1] * requests)


def config3_lengths() -> list:
    gen = torch.Generator().manual_seed(1)
    return [int(x) for x in torch.randint(512, 8193, (8,), generator=gen)]


def config3(seed: int = 0, heads: int = 32, lengths: Optional[list] = None) -> Workload:
    lengths = config3_lengths() if lengths is None else lengths
    torch.manual_seed(seed)
    D = 128
    q, k, v, g, beta = _tokens(sum(lengths), heads, D)
    n = len(lengths)
    pool = torch.zeros(n + 1, heads, D, D).transpose(-1, -2)
    return Workload("cfg3", q, k, v, g, beta, pool, torch.arange(1, n + 1, dtype=torch.int32),
                    _cu(lengths), D ** -0.5, lengths)


def config4(seed: int = 0, heads: int = 32, tokens: int = 131072) -> Workload:
    torch.manual_seed(seed)
    D = 128
    q, k, v, g, beta = _tokens(tokens, heads, D)
    pool = _pool(2, heads, D)
    return Workload("cfg4", q, k, v, g, beta, pool, torch.tensor([1], dtype=torch.int32),
                    _cu([tokens]), D ** -0.5, [tokens])


def config5(seed: int = 0, heads: int = 32, decode: int = 64, prefills: int = 4,
            prefill_len: int = 2048, slots: int = 1024) -> Workload:
    torch.manual_seed(seed)
    D = 128
    lengths = [1] * decode + [prefill_len] * prefills
    q, k, v, g, beta = _tokens(sum(lengths), heads, D)
    pool = _pool(slots, heads, D)
    indices = (torch.randperm(slots - 1)[:len(lengths)] + 1).to(torch.int32)
    return Workload("cfg5", q, k, v, g, beta, pool, indices, _cu(lengths), D ** -0.5, lengths)


def conv_frontend(lengths: list, heads: int = 32, window: int = 3, seed: int = 0, D: int = 128,
                  device: str = "cpu") -> dict:
    """Inputs of one ``kda_causal_conv1d`` call: x [T, 3*H*D], weight [3*H*D, 4],
    conv_state [R + 1, window, 3*H*D], cache_indices, query_start_loc."""
    torch.manual_seed(seed)
    C = 3 * heads * D
    T = sum(lengths)
    d = dict(x=(torch.randn(T, C) * 0.2).bfloat16(), weight=torch.randn(C, 4) * 0.1,
             conv_state=(torch.randn(len(lengths) + 1, window, C) * 0.1).bfloat16(),
             cache_indices=torch.arange(1, len(lengths) + 1, dtype=torch.int32),
             query_start_loc=_cu(lengths))
    return {k: v.to(device) for k, v in d.items()}
