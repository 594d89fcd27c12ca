"""Load the fixtures written by ``tests/golden/make_golden.py``."""

from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def bf16(bits: np.ndarray) -> torch.Tensor:
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz") as z:
        return {k: z[k] for k in z.files}


def kcontig(pool: np.ndarray) -> torch.Tensor:
    """A [slots,H,K,V] pool as the production K-contiguous view."""
    t = torch.from_numpy(pool).float()
    return t.transpose(-1, -2).contiguous().transpose(-1, -2)


def expected_pool(f: dict) -> torch.Tensor:
    """pool_in with the touched slots replaced by the reference's values."""
    pool = torch.from_numpy(f["pool_in"]).float().clone()
    for i, s in enumerate(f["pool_out_slots"].tolist()):
        pool[s] = torch.from_numpy(f["pool_out_vals"][i])
    return pool


def raw_kwargs(f: dict) -> dict:
    """Raw-gate op keyword arguments (CPU tensors) from a fixture."""
    kw = dict(q=bf16(f["q"]), k=bf16(f["k"]), v=bf16(f["v"]), a=bf16(f["a"]),
              b=bf16(f["b"]), A_log=torch.from_numpy(f["A_log"]),
              dt_bias=torch.from_numpy(f["dt_bias"]),
              initial_state_indices=torch.from_numpy(f["indices"]),
              cu_seqlens=torch.from_numpy(f["cu_seqlens"]),
              lower_bound=float(f["lower_bound"]), scale=float(f["scale"]))
    if "track_indices" in f:
        kw["track_state_indices"] = torch.from_numpy(f["track_indices"])
        kw["track_state_lens"] = torch.from_numpy(f["track_lens"])
    return kw
