"""CPU checks of the C ABI boundary (no kernel is launched).

* every function ``include/kda_b200.h`` declares is exported by
  ``libkda_b200.so``;
* the ctypes mirror of ``KdaArgs`` has the header's size and field offsets
  (checked against a tiny C program compiled here with gcc);
* argument validation returns the documented KdaStatus codes before any CUDA
  call is made;
* the sglang plugin hook registers the prepared recurrence.
"""

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "kda_b200.h"


@pytest.fixture(scope="module")
def abi():
    from sgl_glm53_ascend_ops import abi as _abi
    return _abi


def _declared_functions():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kda_[a-z_]+)\s*\(", text)))


def test_header_functions_are_exported(abi):
    lib = abi.lib()
    declared = _declared_functions()
    assert declared, "no declarations parsed"
    assert sorted(abi.EXPORTED) == declared
    for name in declared:
        assert hasattr(lib, name), f"{name} missing from {abi.LIB_PATH.name}"
    assert lib.kda_abi_version() == 1


def test_status_codes_match_header(abi):
    """abi.py's KdaStatus constants are the header's values."""
    codes = dict(re.findall(r"\b(KDA_(?:OK|ERR_[A-Z_]+))\s*=\s*(\d+)", HEADER.read_text()))
    assert len(codes) == 7
    for name, value in codes.items():
        assert getattr(abi, name) == int(value), name


@pytest.mark.parametrize("struct", ["KdaArgs", "KdaCommitArgs", "KdaConvArgs"])
def test_struct_layout_matches_header(abi, tmp_path, struct):
    cls = getattr(abi, struct)
    fields = [f[0] for f in cls._fields_]
    src = ["#include <stdio.h>", "#include <stddef.h>", '#include "kda_b200.h"', "int main(void){",
           f'printf("%zu\\n", sizeof({struct}));']
    src += [f'printf("%zu\\n", offsetof({struct}, {f}));' for f in fields]
    src += ["return 0;}"]
    c = tmp_path / "layout.c"
    c.write_text("\n".join(src))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(c), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], check=True, capture_output=True,
                                           text=True).stdout.split()]
    assert vals[0] == ctypes.sizeof(cls)
    for f, off in zip(fields, vals[1:]):
        assert getattr(cls, f).offset == off, f"offset of {f}"


def test_invalid_arguments_rejected_without_launch(abi):
    lib = abi.lib()
    assert lib.kda_recurrent_launch(None, None) == 1              # KDA_ERR_INVALID_ARGUMENT
    assert lib.kda_prepared_recurrent_launch(None, None) == 1
    assert lib.kda_chunk_launch(None, None, 0, None) == 1
    a = abi.KdaArgs()
    a.head_dim = 96
    a.num_heads = 1
    a.index_bytes[:] = [4, 4, 4, 4]
    assert lib.kda_recurrent_launch(ctypes.byref(a), None) == 2   # KDA_ERR_UNSUPPORTED
    a.head_dim = 128
    a.index_bytes[1] = 3
    assert lib.kda_recurrent_launch(ctypes.byref(a), None) == 1
    a.index_bytes[1] = 4
    a.num_req = 0
    assert lib.kda_recurrent_launch(ctypes.byref(a), None) == 0   # nothing to do, no launch
    a.num_req = 2
    a.head_count = 1
    assert lib.kda_recurrent_launch(ctypes.byref(a), None) == 1   # null pointers
    assert abi.status_string(0x102).startswith("device: state slot")


def test_commit_arguments_rejected_without_launch(abi):
    lib = abi.lib()
    assert lib.kda_commit_intermediate_launch(None, None) == 1
    c = abi.KdaCommitArgs()
    c.index_bytes[:] = [4, 4, 4]
    assert lib.kda_commit_intermediate_launch(ctypes.byref(c), None) == 0     # no entries: nothing to do
    c.num_entries, c.num_layers, c.num_heads, c.head_dim = 2, 1, 4, 128
    assert lib.kda_commit_intermediate_launch(ctypes.byref(c), None) == 1     # null pointers
    c.index_bytes[2] = 2
    assert lib.kda_commit_intermediate_launch(ctypes.byref(c), None) == 1     # bad index width
    c.index_bytes[2] = 4
    c.num_layers = -1
    assert lib.kda_commit_intermediate_launch(ctypes.byref(c), None) == 1


def test_conv_arguments_rejected_without_launch(abi):
    lib = abi.lib()
    assert lib.kda_conv_launch(None, None) == abi.KDA_ERR_INVALID_ARGUMENT
    c = abi.KdaConvArgs()
    c.index_bytes[:] = [4, 4, 1, 4, 4]
    c.channels, c.num_parts, c.width, c.window = 1536, 3, 4, 3
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_OK            # no requests, no tokens: nothing to do
    c.num_tokens = 4
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT   # tokens to zero, null x/out
    c.num_tokens, c.window = 0, 9
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_UNSUPPORTED        # window beyond 8 rows
    c.width = 5
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_UNSUPPORTED
    c.width, c.window = 4, 2
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT   # window < W - 1
    c.window, c.activation = 3, 2
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_UNSUPPORTED
    c.activation, c.num_req = abi.KDA_CONV_ACT_SILU, 2
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT   # null pointers
    c.index_bytes[1] = 2
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT   # bad index width
    c.index_bytes[1] = 4
    buf = (ctypes.c_uint8 * 64)()
    base = (ctypes.addressof(buf) + 15) // 16 * 16
    c.x = c.weight = c.out = c.indices = c.cu_seqlens = c.conv_state = base
    c.x_row_stride, c.state_stride[0], c.state_stride[1] = 1536, 3 * 1536, 1536
    c.num_parts = 5
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT   # parts do not divide C
    c.num_parts, c.channels, c.x_row_stride = 3, 1524, 1524                            # C / 3 = 508: not 8-aligned
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_ALIGNMENT
    c.channels, c.x_row_stride = 1536, 1536
    c.x = base + 2
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_ALIGNMENT
    c.x = base
    c.track_indices = base                                                              # lens missing
    assert lib.kda_conv_launch(ctypes.byref(c), None) == abi.KDA_ERR_INVALID_ARGUMENT


def test_workspace_size_is_queryable(abi):
    n = abi.chunk_workspace_bytes(8, 33494, 32, 128)
    assert n >= 0
    assert abi.chunk_path_workspace_bytes(8, 33494, 32, 128, abi.KDA_CHUNK_AUTO) == n
    fused = abi.chunk_path_workspace_bytes(8, 33494, 32, 128, abi.KDA_CHUNK_FUSED)
    split = abi.chunk_path_workspace_bytes(8, 33494, 32, 128, abi.KDA_CHUNK_SPLIT)
    assert 0 < fused <= 256 < split              # the request order alone vs. per-chunk records
    assert abi.chunk_path_workspace_bytes(8, 33494, 32, 128, 7) == 0
    assert abi.chunk_path_workspace_bytes(2000, 33494, 32, 128, abi.KDA_CHUNK_FUSED) == 0   # > 1024 requests


def test_forced_path_and_selftest_arguments_rejected_without_launch(abi):
    lib = abi.lib()
    a = abi.KdaArgs()
    a.head_dim, a.num_heads = 128, 1
    a.index_bytes[:] = [4, 4, 4, 4]
    assert lib.kda_chunk_launch_path(ctypes.byref(a), None, 0, None, 3) == abi.KDA_ERR_INVALID_ARGUMENT
    assert lib.kda_chunk_launch_path(ctypes.byref(a), None, 0, None, abi.KDA_CHUNK_SPLIT) == abi.KDA_OK  # empty
    a.num_req, a.head_count = 2, 1
    assert lib.kda_chunk_launch_path(ctypes.byref(a), None, 0, None, abi.KDA_CHUNK_SPLIT) == 1   # null pointers
    assert lib.kda_selftest_wait_timeout(None, None, 16, 1, 1, None) == abi.KDA_ERR_INVALID_ARGUMENT


def test_plugin_registers_prepared_recurrent():
    from sgl_glm53_ascend_ops import plugin

    calls = []

    class Registry:
        @staticmethod
        def register(target, fn, hook_type):
            calls.append((target, fn, hook_type))

    plugin.register(Registry)
    assert calls == [(plugin.SGLANG_TARGET_PATH, plugin._prepared_recurrent, "REPLACE")]


def test_ops_registered_with_reference_schemas():
    import torch
    import sgl_glm53_ascend_ops  # noqa: F401

    ns = torch.ops.sgl_glm53_ascend
    rec = str(ns.kda_varlen_recurrent.default._schema)
    assert rec.startswith("sgl_glm53_ascend::kda_varlen_recurrent(*, Tensor A_log, Tensor a, Tensor dt_bias, "
                          "Tensor q, Tensor k, Tensor v, Tensor b, Tensor(a!) initial_state_source")
    assert "Tensor(b!)? intermediate_state=None, bool prefill=False" in rec
    chunk = str(ns.kda_varlen_chunk.default._schema)
    assert "bool prefill=False, Tensor? track_state_indices=None, Tensor? track_state_lens=None) -> Tensor" in chunk
    prep = str(ns.prepared_recurrent.default._schema)
    assert prep.endswith("bool track_state=False, int head_offset=0) -> ()")
    for name in ("kda_varlen_recurrent_v2", "kda_varlen_chunk_v2", "kda_varlen_recurrent_g",
                 "kda_varlen_chunk_g"):
        assert hasattr(ns, name)
    conv = str(ns.kda_causal_conv1d.default._schema)
    assert conv == ("sgl_glm53_ascend::kda_causal_conv1d(Tensor x, Tensor weight, Tensor? bias, "
                    "Tensor(a!) conv_state, Tensor cache_indices, Tensor query_start_loc, "
                    "Tensor? has_initial_state=None, Tensor? track_conv_indices=None, "
                    "Tensor? track_conv_lens=None, int num_parts=3, bool silu=True) -> Tensor")
    commit = str(ns.move_intermediate_cache_kda.default._schema)
    assert commit == ("sgl_glm53_ascend::move_intermediate_cache_kda(Tensor(a!) dst, Tensor src, "
                      "Tensor dst_indices, Tensor src_indices, Tensor step_indices, int h_block_size=1) -> ()")
