"""The chunk prefill through the C ABI with its internal path forced
(``kda_chunk_launch_path``), for the GPU tests: every chunk case runs on the
library's own choice and on the split path, and some also on the fused
kernel or with the kernel's fp32 pre-cast output (``out_fp32``)."""

import torch


def chunk_via_abi(kw: dict, path: int, out_fp32: bool = False) -> torch.Tensor:
    """Run the chunk prefill on the op's keyword arguments (device tensors;
    raw gate when ``a`` is present, else the log gate ``g``/``beta``) through
    ``kda_chunk_launch_path``. Updates the pool in place and returns the
    output: bf16, or fp32 pre-cast values with ``out_fp32``."""
    from sgl_glm53_ascend_ops import abi

    raw = "a" in kw
    v = kw["v"]
    out = torch.empty(v.shape, dtype=torch.float32 if out_fp32 else torch.bfloat16, device=v.device)
    dt = kw.get("dt_bias")
    args = abi.args_from_tensors(
        q=kw["q"], k=kw["k"], v=v, out=out, state=kw["initial_state_source"],
        indices=kw["initial_state_indices"], cu_seqlens=kw["cu_seqlens"], scale=kw["scale"],
        gate_mode=abi.KDA_GATE_RAW if raw else abi.KDA_GATE_LOG, g=kw.get("g"), beta=kw.get("beta"),
        a=kw.get("a"), b=kw.get("b"), A_log=kw.get("A_log"), dt_bias=None if dt is None else dt.contiguous(),
        lower_bound=kw.get("lower_bound", 0.0), track_indices=kw.get("track_state_indices"),
        track_lens=kw.get("track_state_lens"), out_fp32=out_fp32)
    n = abi.chunk_path_workspace_bytes(args.num_req, args.num_tokens, args.head_count, args.head_dim, path)
    ws = torch.empty(max(n, 1), dtype=torch.uint8, device=v.device)
    rc = abi.chunk_launch_path(args, ws, n, path)
    assert rc == abi.KDA_OK, f"kda_chunk_launch_path: {abi.status_string(rc)}"
    torch.cuda.synchronize()
    return out
