"""Find and load ``sgl_glm53_ascend_ops_lib*.so`` (reference: ``_load.py:1-48``)."""

from __future__ import annotations

from pathlib import Path

import torch

_LOADED = False

_LIB_NAME = "sgl_glm53_ascend_ops_lib"


def _find_library() -> Path:
    here = Path(__file__).resolve().parent
    libraries = sorted(here.glob(f"{_LIB_NAME}*.so"))
    if not libraries:
        raise RuntimeError(
            f"Cannot find {_LIB_NAME}*.so in {here}. "
            "Run 'python 01-glm53-ascend_b200/build.py' to build the library."
        )
    return libraries[0]


def load_library() -> None:
    global _LOADED
    if _LOADED:
        return
    torch.ops.load_library(str(_find_library()))
    _LOADED = True
