"""GLM-5.3 KDA operator extensions for SGLang, built for NVIDIA B200 (sm_100a).

Importing the package loads the compiled torch-op library (same behaviour as
the reference's ``sgl_glm53_ascend_ops/__init__.py:1-5``); there is no CPU or
Python fallback, so a missing build raises here.
"""

from ._load import load_library

load_library()
