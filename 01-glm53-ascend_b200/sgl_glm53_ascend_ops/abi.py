"""ctypes binding of the C ABI in ``include/kda_b200.h`` (``libkda_b200.so``).

This is the binding a non-torch host (or a maintainer wiring the library into
another runtime) would write: a ``KdaArgs`` struct of raw device pointers,
strides and sizes, and the launch entry points. ``args_from_tensors``
fills the struct from torch tensors for tests and the benchmark; the library
itself never sees a torch type.
"""

from __future__ import annotations

import ctypes
from pathlib import Path
from typing import Optional

import torch

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "libkda_b200.so"

KDA_OK = 0
# KdaStatus (include/kda_b200.h)
(KDA_ERR_INVALID_ARGUMENT, KDA_ERR_UNSUPPORTED, KDA_ERR_ALIGNMENT, KDA_ERR_WORKSPACE, KDA_ERR_LAUNCH,
 KDA_ERR_TOO_LARGE) = range(1, 7)
KDA_GATE_RAW, KDA_GATE_LOG, KDA_GATE_PREPARED = 0, 1, 2
KDA_CHUNK_AUTO, KDA_CHUNK_FUSED, KDA_CHUNK_SPLIT = 0, 1, 2
KDA_CONV_ACT_NONE, KDA_CONV_ACT_SILU = 0, 1

# Entry points declared in include/kda_b200.h.
EXPORTED = (
    "kda_abi_version",
    "kda_status_string",
    "kda_recurrent_launch",
    "kda_chunk_workspace_bytes",
    "kda_chunk_launch",
    "kda_chunk_launch_phases",
    "kda_chunk_launch_path",
    "kda_chunk_path_workspace_bytes",
    "kda_prepared_recurrent_launch",
    "kda_chunk_launch_no_alloc",
    "kda_commit_intermediate_launch",
    "kda_selftest_wait_timeout",
    "kda_conv_launch",
)


class KdaArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p),
        ("k", ctypes.c_void_p),
        ("v", ctypes.c_void_p),
        ("a", ctypes.c_void_p),
        ("b", ctypes.c_void_p),
        ("A_log", ctypes.c_void_p),
        ("dt_bias", ctypes.c_void_p),
        ("g", ctypes.c_void_p),
        ("beta", ctypes.c_void_p),
        ("out", ctypes.c_void_p),
        ("state", ctypes.c_void_p),
        ("state_stride", ctypes.c_int64 * 4),
        ("num_slots", ctypes.c_int64),
        ("indices", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("track_indices", ctypes.c_void_p),
        ("track_lens", ctypes.c_void_p),
        ("intermediate", ctypes.c_void_p),
        ("mid_stride", ctypes.c_int64 * 5),
        ("index_bytes", ctypes.c_int32 * 4),
        ("num_req", ctypes.c_int32),
        ("num_tokens", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("head_begin", ctypes.c_int32),
        ("head_count", ctypes.c_int32),
        ("gate_mode", ctypes.c_int32),
        ("scale", ctypes.c_float),
        ("lower_bound", ctypes.c_float),
        ("status", ctypes.c_void_p),
        ("out_fp32", ctypes.c_int32),
    ]


class KdaCommitArgs(ctypes.Structure):
    _fields_ = [
        ("dst", ctypes.c_void_p),
        ("src", ctypes.c_void_p),
        ("dst_stride", ctypes.c_int64 * 5),
        ("src_stride", ctypes.c_int64 * 6),
        ("dst_indices", ctypes.c_void_p),
        ("src_indices", ctypes.c_void_p),
        ("step_indices", ctypes.c_void_p),
        ("index_bytes", ctypes.c_int32 * 3),
        ("num_entries", ctypes.c_int32),
        ("num_layers", ctypes.c_int32),
        ("num_heads", ctypes.c_int32),
        ("head_dim", ctypes.c_int32),
        ("num_slots", ctypes.c_int64),
        ("num_requests", ctypes.c_int32),
        ("num_steps", ctypes.c_int32),
        ("status", ctypes.c_void_p),
    ]


class KdaConvArgs(ctypes.Structure):
    _fields_ = [
        ("x", ctypes.c_void_p),
        ("x_row_stride", ctypes.c_int64),
        ("weight", ctypes.c_void_p),
        ("bias", ctypes.c_void_p),
        ("conv_state", ctypes.c_void_p),
        ("state_stride", ctypes.c_int64 * 2),
        ("num_slots", ctypes.c_int64),
        ("window", ctypes.c_int32),
        ("indices", ctypes.c_void_p),
        ("cu_seqlens", ctypes.c_void_p),
        ("has_initial", ctypes.c_void_p),
        ("track_indices", ctypes.c_void_p),
        ("track_lens", ctypes.c_void_p),
        ("index_bytes", ctypes.c_int32 * 5),
        ("num_req", ctypes.c_int32),
        ("num_tokens", ctypes.c_int32),
        ("channels", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("num_parts", ctypes.c_int32),
        ("activation", ctypes.c_int32),
        ("out", ctypes.c_void_p),
        ("status", ctypes.c_void_p),
    ]


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(f"{LIB_PATH} is missing; run 01-glm53-ascend_b200/build.py")
        L = ctypes.CDLL(str(LIB_PATH))
        L.kda_abi_version.restype = ctypes.c_int
        L.kda_status_string.restype = ctypes.c_char_p
        L.kda_status_string.argtypes = [ctypes.c_int]
        for name in ("kda_recurrent_launch", "kda_prepared_recurrent_launch"):
            getattr(L, name).restype = ctypes.c_int
            getattr(L, name).argtypes = [ctypes.POINTER(KdaArgs), ctypes.c_void_p]
        L.kda_chunk_workspace_bytes.restype = ctypes.c_size_t
        L.kda_chunk_workspace_bytes.argtypes = [ctypes.c_int32] * 4
        L.kda_chunk_launch_no_alloc.restype = ctypes.c_int
        L.kda_chunk_launch_no_alloc.argtypes = [ctypes.POINTER(KdaArgs), ctypes.c_void_p]
        L.kda_commit_intermediate_launch.restype = ctypes.c_int
        L.kda_commit_intermediate_launch.argtypes = [ctypes.POINTER(KdaCommitArgs), ctypes.c_void_p]
        L.kda_chunk_launch.restype = ctypes.c_int
        L.kda_chunk_launch.argtypes = [ctypes.POINTER(KdaArgs), ctypes.c_void_p, ctypes.c_size_t,
                                       ctypes.c_void_p]
        L.kda_chunk_launch_path.restype = ctypes.c_int
        L.kda_chunk_launch_path.argtypes = [ctypes.POINTER(KdaArgs), ctypes.c_void_p, ctypes.c_size_t,
                                            ctypes.c_void_p, ctypes.c_int32]
        L.kda_chunk_path_workspace_bytes.restype = ctypes.c_size_t
        L.kda_chunk_path_workspace_bytes.argtypes = [ctypes.c_int32] * 5
        L.kda_selftest_wait_timeout.restype = ctypes.c_int
        L.kda_selftest_wait_timeout.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int32, ctypes.c_int32,
                                                ctypes.c_int32, ctypes.c_void_p]
        L.kda_conv_launch.restype = ctypes.c_int
        L.kda_conv_launch.argtypes = [ctypes.POINTER(KdaConvArgs), ctypes.c_void_p]
        L.kda_chunk_launch_phases.restype = ctypes.c_int
        L.kda_chunk_launch_phases.argtypes = [ctypes.POINTER(KdaArgs), ctypes.c_void_p, ctypes.c_size_t,
                                              ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), ctypes.c_int]
        _lib = L
    return _lib


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _ibytes(t: Optional[torch.Tensor]) -> int:
    return 8 if (t is not None and t.dtype == torch.int64) else 4


def args_from_tensors(*, q, k, v, out, state, indices, cu_seqlens, scale, gate_mode,
                      g=None, beta=None, a=None, b=None, A_log=None, dt_bias=None,
                      lower_bound=0.0, track_indices=None, track_lens=None,
                      intermediate=None, head_begin=0, head_count=None,
                      status=None, out_fp32=False) -> KdaArgs:
    """Fill KdaArgs from device tensors ([1,T,H,D] token tensors, [slots,H,K,V] pool)."""
    H, D = state.shape[1], state.shape[2]
    T = q.numel() // (H * D)
    x = KdaArgs()
    x.q, x.k, x.v, x.out = _ptr(q), _ptr(k), _ptr(v), _ptr(out)
    x.a, x.b, x.A_log, x.dt_bias = _ptr(a), _ptr(b), _ptr(A_log), _ptr(dt_bias)
    x.g, x.beta = _ptr(g), _ptr(beta)
    x.state = _ptr(state)
    for i in range(4):
        x.state_stride[i] = state.stride(i)
    x.num_slots = state.shape[0]
    x.indices, x.cu_seqlens = _ptr(indices), _ptr(cu_seqlens)
    x.track_indices, x.track_lens = _ptr(track_indices), _ptr(track_lens)
    x.intermediate = _ptr(intermediate)
    if intermediate is not None:
        for i in range(5):
            x.mid_stride[i] = intermediate.stride(i)
    for i, t in enumerate((indices, cu_seqlens, track_indices, track_lens)):
        x.index_bytes[i] = _ibytes(t)
    x.num_req = indices.numel()
    x.num_tokens = T
    x.num_heads = H
    x.head_dim = D
    x.head_begin = head_begin
    x.head_count = H - head_begin if head_count is None else head_count
    x.gate_mode = gate_mode
    x.scale = float(scale)
    x.lower_bound = float(lower_bound)
    x.status = _ptr(status)
    x.out_fp32 = int(bool(out_fp32))
    return x


def stream_handle(stream: Optional[torch.cuda.Stream] = None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream


def recurrent_launch(args: KdaArgs, stream: Optional[torch.cuda.Stream] = None) -> int:
    return lib().kda_recurrent_launch(ctypes.byref(args), stream_handle(stream))


def prepared_recurrent_launch(args: KdaArgs, stream: Optional[torch.cuda.Stream] = None) -> int:
    return lib().kda_prepared_recurrent_launch(ctypes.byref(args), stream_handle(stream))


def chunk_workspace_bytes(num_req: int, num_tokens: int, num_heads: int, head_dim: int) -> int:
    return lib().kda_chunk_workspace_bytes(num_req, num_tokens, num_heads, head_dim)


def chunk_launch(args: KdaArgs, workspace: Optional[torch.Tensor], workspace_bytes: int,
                 stream: Optional[torch.cuda.Stream] = None) -> int:
    return lib().kda_chunk_launch(ctypes.byref(args), _ptr(workspace), workspace_bytes,
                                  stream_handle(stream))


def chunk_path_workspace_bytes(num_req: int, num_tokens: int, num_heads: int, head_dim: int, path: int) -> int:
    return lib().kda_chunk_path_workspace_bytes(num_req, num_tokens, num_heads, head_dim, path)


def chunk_launch_path(args: KdaArgs, workspace: Optional[torch.Tensor], workspace_bytes: int, path: int,
                      stream: Optional[torch.cuda.Stream] = None) -> int:
    """kda_chunk_launch with the internal path forced (KDA_CHUNK_AUTO/FUSED/SPLIT)."""
    return lib().kda_chunk_launch_path(ctypes.byref(args), _ptr(workspace), workspace_bytes,
                                       stream_handle(stream), path)


def chunk_launch_phases(args: KdaArgs, workspace: torch.Tensor, workspace_bytes: int, events,
                        stream: Optional[torch.cuda.Stream] = None) -> int:
    """kda_chunk_launch's split path with six torch.cuda.Events (timing
    enabled, each recorded once before) marking its phases: before the plan,
    after prep, the scan's first pass, the combine, the rescan, the outputs."""
    handles = (ctypes.c_void_p * 6)(*[ctypes.c_void_p(e.cuda_event) for e in events])
    return lib().kda_chunk_launch_phases(ctypes.byref(args), _ptr(workspace), workspace_bytes,
                                         stream_handle(stream), handles, len(events))


def chunk_launch_no_alloc(args: KdaArgs, stream: Optional[torch.cuda.Stream] = None) -> int:
    """kda_chunk_launch without a caller workspace (scratch inside the library)."""
    return lib().kda_chunk_launch_no_alloc(ctypes.byref(args), stream_handle(stream))


def commit_args_from_tensors(dst, src, dst_indices, src_indices, step_indices,
                             status: Optional[torch.Tensor] = None) -> KdaCommitArgs:
    """dst [layers, slots, H, D, D] fp32, src [layers, requests, steps, H, D, D] fp32."""
    x = KdaCommitArgs()
    x.dst, x.src = dst.data_ptr(), src.data_ptr()
    for i in range(5):
        x.dst_stride[i] = dst.stride(i)
    for i in range(6):
        x.src_stride[i] = src.stride(i)
    x.dst_indices, x.src_indices, x.step_indices = (t.data_ptr() for t in (dst_indices, src_indices, step_indices))
    for i, t in enumerate((dst_indices, src_indices, step_indices)):
        x.index_bytes[i] = _ibytes(t)
    x.num_entries = dst_indices.numel()
    x.num_layers, x.num_slots, x.num_heads, x.head_dim = dst.shape[0], dst.shape[1], dst.shape[2], dst.shape[3]
    x.num_requests, x.num_steps = src.shape[1], src.shape[2]
    x.status = _ptr(status)
    return x


def commit_launch(args: KdaCommitArgs, stream: Optional[torch.cuda.Stream] = None) -> int:
    return lib().kda_commit_intermediate_launch(ctypes.byref(args), stream_handle(stream))


def selftest_wait_timeout(status: torch.Tensor, expired: torch.Tensor, polls: int, waits: int, give_up: bool,
                          stream: Optional[torch.cuda.Stream] = None) -> int:
    """Waits that must run out (see kda_selftest_wait_timeout in the header)."""
    return lib().kda_selftest_wait_timeout(_ptr(status), _ptr(expired), polls, waits, int(give_up),
                                           stream_handle(stream))


def conv_args_from_tensors(*, x, weight, conv_state, indices, cu_seqlens, out, bias=None, has_initial=None,
                           track_indices=None, track_lens=None, num_parts=3, silu=True,
                           status=None) -> KdaConvArgs:
    """KdaConvArgs from device tensors: x [T, C] bf16 (channel-contiguous rows),
    weight [C, W] fp32 contiguous, conv_state [slots, window, C] bf16
    (channel-contiguous), out [num_parts, T, C / num_parts] bf16."""
    a = KdaConvArgs()
    a.x, a.x_row_stride = _ptr(x), x.stride(0)
    a.weight, a.bias = _ptr(weight), _ptr(bias)
    a.conv_state = _ptr(conv_state)
    a.state_stride[0], a.state_stride[1] = conv_state.stride(0), conv_state.stride(1)
    a.num_slots, a.window = conv_state.shape[0], conv_state.shape[1]
    a.indices, a.cu_seqlens, a.has_initial = _ptr(indices), _ptr(cu_seqlens), _ptr(has_initial)
    a.track_indices, a.track_lens = _ptr(track_indices), _ptr(track_lens)
    a.index_bytes[0], a.index_bytes[1] = _ibytes(indices), _ibytes(cu_seqlens)
    a.index_bytes[2] = has_initial.element_size() if has_initial is not None else 1
    a.index_bytes[3], a.index_bytes[4] = _ibytes(track_indices), _ibytes(track_lens)
    a.num_req, a.num_tokens = indices.numel(), x.shape[0]
    a.channels, a.width = x.shape[1], weight.shape[1]
    a.num_parts = num_parts
    a.activation = KDA_CONV_ACT_SILU if silu else KDA_CONV_ACT_NONE
    a.out = _ptr(out)
    a.status = _ptr(status)
    return a


def conv_launch(args: KdaConvArgs, stream: Optional[torch.cuda.Stream] = None) -> int:
    return lib().kda_conv_launch(ctypes.byref(args), stream_handle(stream))


def status_string(code: int) -> str:
    return lib().kda_status_string(code).decode()
