"""Build the B200 KDA extension in-tree (no JIT cache, nothing installed).

Produces, inside ``sgl_glm53_ascend_ops/``:

* ``libkda_b200.so`` -- the CUDA kernels and the C ABI of ``include/kda_b200.h``
  (nvcc, ``-gencode arch=compute_100a,code=sm_100a``, static cudart);
* ``sgl_glm53_ascend_ops_lib.so`` -- the torch ops (``torch_ops.cpp``), linked
  against ``libkda_b200.so`` with an ``$ORIGIN`` rpath. The name matches the
  reference loader's ``sgl_glm53_ascend_ops_lib*.so`` pattern.

Run ``python 01-glm53-ascend_b200/build.py`` (add ``--force`` to rebuild).
Each step is skipped when its output is newer than all of its inputs.
"""

from __future__ import annotations

import os
import subprocess
import sys
import sysconfig
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
CSRC = HERE / "csrc"
INCLUDE = ROOT / "include"
OUT = HERE / "sgl_glm53_ascend_ops"
KERNEL_LIB = OUT / "libkda_b200.so"
OPS_LIB = OUT / "sgl_glm53_ascend_ops_lib.so"
CUDA_HOME = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def _run(cmd):
    print("+", " ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def build_kernels(force: bool = False) -> Path:
    sources = sorted(CSRC.glob("*.cu"))
    deps = sources + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "kda_b200.h"]
    if force or _stale(KERNEL_LIB, deps):
        objs = []
        build_dir = HERE / "_build"
        build_dir.mkdir(exist_ok=True)
        for src in sources:
            obj = build_dir / (src.stem + ".o")
            _run([CUDA_HOME / "bin" / "nvcc", *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
                  "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj])
            objs.append(obj)
        _run([CUDA_HOME / "bin" / "nvcc", *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", KERNEL_LIB])
    return KERNEL_LIB


def build_ops(force: bool = False) -> Path:
    import torch
    from torch.utils import cpp_extension

    src = CSRC / "torch_ops.cpp"
    deps = [src, INCLUDE / "kda_b200.h", KERNEL_LIB]
    if force or _stale(OPS_LIB, deps):
        incs = cpp_extension.include_paths(device_type="cuda") + [str(CUDA_HOME / "include"), str(INCLUDE),
                                                                  sysconfig.get_paths()["include"]]
        libdirs = cpp_extension.library_paths(device_type="cuda")
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        cmd = ["g++", "-O2", "-std=c++17", "-shared", "-fPIC", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-DTORCH_EXTENSION_NAME=sgl_glm53_ascend_ops_lib", "-DTORCH_API_INCLUDE_EXTENSION_H"]
        cmd += [f"-I{p}" for p in incs]
        cmd += [str(src), "-o", str(OPS_LIB), f"-L{OUT}", "-lkda_b200", "-Wl,-rpath,$ORIGIN"]
        cmd += [f"-L{p}" for p in libdirs] + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda"]
        cmd += [f"-Wl,-rpath,{p}" for p in libdirs]
        _run(cmd)
    return OPS_LIB


def build(force: bool = False) -> None:
    build_kernels(force)
    build_ops(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
