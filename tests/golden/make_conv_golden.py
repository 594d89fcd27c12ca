"""Generate the fixtures that pin ``oracle/conv_ref.py`` to a published causal conv1d.

sglang's causal-conv code (the front end of the reference's attention backend)
is in neither the reference tree nor this image. The algorithm it implements is
the causal-conv1d one (Dao-AILab ``causal_conv1d_fn``), of which vLLM 0.22
ships a plain-torch CPU restatement, ``causal_conv1d_torch`` in
``vllm/model_executor/layers/mamba/ops/cpu/causal_conv1d.py``. This script runs
that function on seeded inputs and stores inputs and outputs; the oracle is
checked against them by ``tests/test_conv_cpu.py``.

Run where vLLM is installed (it is not needed at test time):

    python tests/golden/make_conv_golden.py

The module file is loaded on its own (it imports only torch), so vLLM's
package initialisation does not run. vLLM's layout is channel-major
(x [C, T], conv_states [slots, C, W - 1]); the fixtures store the operator's
time-major layout (x [T, C], conv state [slots, W - 1, C]). Both cases keep
the state window at W - 1 rows, the window vLLM's function maintains.

Fixtures store bf16 tensors as raw uint16 bits.
"""

from __future__ import annotations

import importlib.metadata
import importlib.util
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _find_vllm_conv():
    """Locate vLLM's file without importing the vllm package."""
    spec = importlib.util.find_spec("vllm")
    if spec is None or spec.origin is None:
        raise SystemExit("vLLM is not installed here")
    path = Path(spec.origin).resolve().parent / "model_executor/layers/mamba/ops/cpu/causal_conv1d.py"
    mspec = importlib.util.spec_from_file_location("vllm_cpu_causal_conv1d", path)
    mod = importlib.util.module_from_spec(mspec)
    mspec.loader.exec_module(mod)
    return mod.causal_conv1d_torch


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_case(name, lengths, C, W, slots, slot_ids, has_init, activation, bias, seed):
    conv = _find_vllm_conv()
    g = torch.Generator().manual_seed(seed)
    T = sum(lengths)
    x = (torch.randn(T, C, generator=g) * 0.5).bfloat16()
    weight = torch.randn(C, W, generator=g) * 0.3
    b = torch.randn(C, generator=g) * 0.1 if bias else None
    state = (torch.randn(slots, W - 1, C, generator=g) * 0.5).bfloat16()
    cu = torch.tensor([0] + list(np.cumsum(lengths)), dtype=torch.int32)
    idx = torch.tensor(slot_ids, dtype=torch.int32)
    init = torch.tensor(has_init, dtype=torch.bool)

    # vLLM layout: x [C, T], conv_states [slots, C, W - 1]
    states_v = state.transpose(1, 2).contiguous()
    out_v = conv(x.t().contiguous(), weight, b, states_v, cu, idx, init, activation=activation)
    fixture = dict(
        x=_bits(x), weight=weight.numpy(), state_in=_bits(state), cu_seqlens=cu.numpy(),
        indices=idx.numpy(), has_initial=init.numpy(), activation=np.array(activation or "none"),
        out=_bits(out_v.t().contiguous()), state_out=_bits(states_v.transpose(1, 2).contiguous()),
        source=np.array(f"vllm {importlib.metadata.version('vllm')} causal_conv1d_torch"),
    )
    if b is not None:
        fixture["bias"] = b.numpy()
    np.savez_compressed(HERE / f"{name}.npz", **fixture)
    print("wrote", name, "T", T, "C", C, "W", W)


def main():
    # Mixed continuing / fresh requests, lengths below, at and above W, no activation
    # (the conv itself, one rounding) and with SiLU (vLLM rounds the conv to bf16
    # before its SiLU; the operator rounds once, so outputs may differ by an ulp).
    make_case("conv_vllm_linear", [5, 1, 3, 17, 2, 9], C=64, W=4, slots=9, slot_ids=[3, 5, 1, 7, 2, 8],
              has_init=[True, True, False, True, False, True], activation=None, bias=True, seed=11)
    make_case("conv_vllm_silu", [7, 4, 1, 30], C=96, W=4, slots=6, slot_ids=[2, 4, 5, 1],
              has_init=[False, True, True, True], activation="silu", bias=False, seed=12)
    make_case("conv_vllm_w3", [6, 2, 11], C=32, W=3, slots=5, slot_ids=[4, 1, 2],
              has_init=[True, False, True], activation="silu", bias=True, seed=13)


if __name__ == "__main__":
    main()
