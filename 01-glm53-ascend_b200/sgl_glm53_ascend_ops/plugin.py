"""sglang plugin entry point (reference: ``plugin.py:1-34``, ``pyproject.toml:12-13``).

``register()`` is what sglang's plugin loader calls for the
``sglang.srt.plugins`` entry-point group. It installs ``prepared_recurrent`` as
a REPLACE hook; the target path is the reference's placeholder string, which a
deployment sets to the sglang function it replaces. sglang is imported lazily
so the package loads without it.
"""

from typing import Optional

import torch

SGLANG_TARGET_PATH = "SGLANG_TARGET_PATH"


def _prepared_recurrent(
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
    from .ops.kda import prepared_recurrent

    return prepared_recurrent(
        qn, kn, v, gdecay, beta, out, state, indices, starts,
        track_indices, track_lens, track_state, head_offset,
    )


def register(registry=None) -> None:
    """Register the hook with sglang's ``HookRegistry`` (or ``registry``, any
    object with the same ``register(target, fn, hook_type)`` method)."""
    if registry is None:
        from sglang.srt.plugins.hook_registry import HookRegistry, HookType

        registry, replace = HookRegistry, HookType.REPLACE
    else:
        replace = "REPLACE"
    registry.register(SGLANG_TARGET_PATH, _prepared_recurrent, replace)
