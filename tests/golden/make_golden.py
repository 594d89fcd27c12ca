"""Generate the golden fixtures that pin ``oracle/kda_ref.py`` to the reference.

Run here, where the reference checkout is readable (it is NOT present on the GPU
box, so nothing at test time imports it):

    REF_ROOT=<reference checkout> python tests/golden/make_golden.py

Each fixture is produced by the reference's own code on seeded CPU inputs:

* ``kda_recur_torch`` and ``kda_chunk_torch`` from ``bench/kda_chunk/kda_python.py``,
  imported with a stub ``torch_npu`` module (the file imports it only to
  register the NPU device). ``kda_recur_torch`` is called once per sequence
  with ``cu_seqlens = [0, len]``: its packed indexing is only correct at
  ``bos == 0`` (kda_python.py:271-303).
* ``_reference`` from ``sgl-glm53-ascend-ops/tests/ops/test_kda_chunk.py``
  (its in-file fp32 transcription), with the module's ``DEVICE`` set to cpu and
  ``D`` to 64 to keep the fixtures small.
* the Triton ``_prepared_recurrent`` from
  ``bench/_prepared_recurrent/bench_prepared_recurrent.py`` under
  ``TRITON_INTERPRET=1`` (the CPU interpreter).

For the prepared-gate (log-decay) cases the reference prologue
``kda_pre_torch`` is wrapped so the norms come from the reference and g/beta are
the injected values: the recurrence itself is the reference's.

Fixtures store bf16 tensors as raw uint16 bits and everything else as float32 or
int64 arrays.
"""

from __future__ import annotations

import os
import sys
import types
from pathlib import Path

os.environ.setdefault("TRITON_INTERPRET", "1")

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
# The reference checkout: given by the caller, never assumed.
REF_ROOT = Path(os.environ["REF_ROOT"]) if os.environ.get("REF_ROOT") else None


def _stub(name, **attrs):
    mod = types.ModuleType(name)
    for k, v in attrs.items():
        setattr(mod, k, v)
    sys.modules[name] = mod
    return mod


def _load_reference():
    if REF_ROOT is None or not REF_ROOT.is_dir():
        raise SystemExit("set REF_ROOT to the reference checkout (the directory holding bench/ and "
                         "sgl-glm53-ascend-ops/)")
    _stub("torch_npu")
    pkg = _stub("sgl_glm53_ascend_ops")
    pkg.__path__ = []
    _stub("sgl_glm53_ascend_ops.ops", kda_varlen_chunk=None, prepared_recurrent=None)
    _stub("benchmark", benchmark=None, BenchmarkConfig=None, print_results_table=None,
          NpuEventMeasurer=None, Reference=None)
    sys.path.insert(0, str(REF_ROOT / "bench" / "kda_chunk"))
    sys.path.insert(0, str(REF_ROOT / "bench" / "_prepared_recurrent"))
    sys.path.insert(0, str(REF_ROOT / "sgl-glm53-ascend-ops" / "tests" / "ops"))
    import kda_python  # noqa: E402
    import test_kda_chunk  # noqa: E402
    import bench_prepared_recurrent  # noqa: E402
    test_kda_chunk.DEVICE = "cpu"
    test_kda_chunk.D = 64
    test_kda_chunk.SLOTS = 5
    return kda_python, test_kda_chunk, bench_prepared_recurrent


def _bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).contiguous().view(torch.int16).numpy().view(np.uint16)


def _f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().contiguous().numpy()


def _kcontig_pool(slots, H, D, scale=0.1):
    """[slots,H,K,V] view of a [slots,H,V,K] allocation (stride(2) == 1)."""
    return (torch.randn(slots, H, D, D) * scale).transpose(-1, -2)


def _touched(pool_in, pool_out):
    """Only the slots a call wrote: (slot list, their values)."""
    diff = (pool_in != pool_out).reshape(pool_in.shape[0], -1).any(1)
    slots = [int(i) for i in torch.nonzero(diff).flatten()]
    return np.array(slots, dtype=np.int64), _f32(pool_out[slots])


def _save(name, **arrays):
    if "pool_out" in arrays and "pool_in" in arrays:
        pin = torch.from_numpy(arrays["pool_in"])
        pout = torch.from_numpy(arrays.pop("pool_out"))
        arrays["pool_out_slots"], arrays["pool_out_vals"] = _touched(pin, pout)
    np.savez_compressed(HERE / f"{name}.npz", **arrays)
    size = (HERE / f"{name}.npz").stat().st_size
    print(f"{name}: {size / 1024:.0f} KiB")


def _per_sequence_recur(kp, kw, cu, slots, intermediate=None):
    """kda_recur_torch one sequence at a time (it is correct at bos == 0)."""
    outs = []
    for i in range(len(cu) - 1):
        bos, eos = cu[i], cu[i + 1]
        sub = dict(kw)
        for n in ("q", "k", "v", "a", "b"):
            sub[n] = kw[n][:, bos:eos]
        sub["initial_state_indices"] = torch.tensor([slots[i]])
        sub["cu_seqlens"] = torch.tensor([0, eos - bos])
        if intermediate is not None:
            sub["intermediate_state"] = intermediate[i:i + 1]
        outs.append(kp.kda_recur_torch(**sub))
    return torch.cat(outs, 1)


def _with_log_gate(kp, g, beta):
    """Wrap kda_pre_torch so the reference norms meet an injected g/beta."""
    original = kp.kda_pre_torch

    def pre(A_log, a, dt_bias, q, k, b, lower_bound, scale):
        qn, kn, _, _ = original(A_log, a, dt_bias, q, k, b, lower_bound, scale)
        sl = getattr(pre, "slice", slice(None))
        return qn, kn, g[:, sl], beta[:, sl]

    return original, pre


def cfg1(kp):
    """cu=[0,37,128], H=4, K=V=64, log gate, seed 0."""
    torch.manual_seed(0)
    T, H, D = 128, 4, 64
    cu = [0, 37, 128]
    q, k, v = (torch.randn(1, T, H, D).bfloat16().float() for _ in range(3))
    g = torch.nn.functional.logsigmoid(torch.randn(1, T, H, D)).clamp(-5.0, 0.0)
    beta = torch.sigmoid(torch.randn(1, T, H))
    init = torch.randn(2, H, D, D) * 0.1
    pool = torch.zeros(3, H, D, D).transpose(-1, -2).contiguous().transpose(-1, -2)
    pool[1:] = init
    pool_in = pool.clone()
    original, pre = _with_log_gate(kp, g, beta)
    kp.kda_pre_torch = pre
    try:
        outs = []
        for i, slot in enumerate((1, 2)):
            bos, eos = cu[i], cu[i + 1]
            pre.slice = slice(bos, eos)
            outs.append(kp.kda_recur_torch(
                A_log=torch.zeros(H), a=torch.zeros(1, eos - bos, H, D),
                dt_bias=torch.zeros(H, D), q=q[:, bos:eos], k=k[:, bos:eos],
                v=v[:, bos:eos], b=torch.zeros(1, eos - bos, H),
                initial_state_source=pool, initial_state_indices=torch.tensor([slot]),
                cu_seqlens=torch.tensor([0, eos - bos]), lower_bound=-5.0,
                scale=D ** -0.5))
    finally:
        kp.kda_pre_torch = original
    out = torch.cat(outs, 1)
    _save("cfg1_recurrent_loggate", q=_bf16_bits(q), k=_bf16_bits(k), v=_bf16_bits(v),
          g=_f32(g), beta=_f32(beta), pool_in=_f32(pool_in), pool_out=_f32(pool),
          indices=np.array([1, 2]), cu_seqlens=np.array(cu), scale=np.float32(D ** -0.5),
          out=_f32(out))


def _raw_inputs(T, H, D, seed):
    torch.manual_seed(seed)
    t = {n: (torch.randn(1, T, H, D) * 0.2).bfloat16() for n in ("q", "k", "v", "a")}
    t["b"] = torch.randn(1, T, H).bfloat16()
    t["A_log"] = torch.randn(H) * 0.1
    t["dt_bias"] = torch.randn(H, D) * 0.1
    return t


def _raw_arrays(t):
    return dict(q=_bf16_bits(t["q"]), k=_bf16_bits(t["k"]), v=_bf16_bits(t["v"]),
                a=_bf16_bits(t["a"]), b=_bf16_bits(t["b"]), A_log=_f32(t["A_log"]),
                dt_bias=_f32(t["dt_bias"]))


def recur_raw_tracked(kp, D, H, T, name, seed):
    """kda_recur_torch, raw gate, one sequence, slot 2, track 20 tokens -> 3."""
    t = _raw_inputs(T, H, D, seed)
    pool = _kcontig_pool(4, H, D)
    pool_in = pool.clone()
    kw = dict(t, initial_state_source=pool, initial_state_indices=torch.tensor([2]),
              cu_seqlens=torch.tensor([0, T]), lower_bound=-5.0, scale=D ** -0.5,
              track_state_indices=torch.tensor([3]), track_state_lens=torch.tensor([20]))
    out = kp.kda_recur_torch(**kw)
    _save(name, **_raw_arrays(t), pool_in=_f32(pool_in), pool_out=_f32(pool),
          indices=np.array([2]), cu_seqlens=np.array([0, T]), track_indices=np.array([3]),
          track_lens=np.array([20]), lower_bound=np.float32(-5.0),
          scale=np.float32(D ** -0.5), out=_f32(out.float()))


def recur_raw_varlen_intermediate(kp):
    """Verify-style per-step checkpoints: lengths [4,3,4], slots [2,0,1]."""
    D, H = 64, 1
    lens, slots = [4, 3, 4], [2, 0, 1]
    cu = [0, 4, 7, 11]
    t = _raw_inputs(cu[-1], H, D, 7)
    pool = _kcontig_pool(3, H, D)
    pool_in = pool.clone()
    torch.manual_seed(5150)
    mid = (torch.randn(3, 4, H, D, D) * 0.1).transpose(-1, -2)
    kw = dict(t, initial_state_source=pool, lower_bound=-5.0, scale=D ** -0.5)
    out = _per_sequence_recur(kp, kw, cu, slots, intermediate=mid)
    _save("recur_raw_intermediate", **_raw_arrays(t), pool_in=_f32(pool_in),
          pool_out=_f32(pool), mid_out_rows=np.array([0, 2]), mid_out=_f32(mid[[0, 2]]),
          indices=np.array(slots), cu_seqlens=np.array(cu), lower_bound=np.float32(-5.0),
          scale=np.float32(D ** -0.5), out=_f32(out.float()))


def recur_raw_varlen(kp):
    """Several sequences, including slot 0, through per-sequence calls."""
    D, H = 64, 2
    cu, slots = [0, 1, 6, 6, 19], [3, 1, 2, 0]
    t = _raw_inputs(cu[-1], H, D, 11)
    pool = _kcontig_pool(4, H, D)
    pool_in = pool.clone()
    kw = dict(t, initial_state_source=pool, lower_bound=-5.0, scale=D ** -0.5)
    out = _per_sequence_recur(kp, kw, cu, slots)
    _save("recur_raw_varlen", **_raw_arrays(t), pool_in=_f32(pool_in), pool_out=_f32(pool),
          indices=np.array(slots), cu_seqlens=np.array(cu), lower_bound=np.float32(-5.0),
          scale=np.float32(D ** -0.5), out=_f32(out.float()))


def chunk_raw(kp):
    """kda_chunk_torch: two aligned sequences, tracked mid-chunk."""
    D, H = 64, 2
    cu, slots = [0, 64, 128], [1, 2]
    t = _raw_inputs(cu[-1], H, D, 3)
    pool = _kcontig_pool(4, H, D)
    pool_in = pool.clone()
    kw = dict(t, initial_state_source=pool, initial_state_indices=torch.tensor(slots),
              cu_seqlens=torch.tensor(cu), lower_bound=-5.0, chunk_size=64,
              scale=D ** -0.5, track_state_indices=torch.tensor([3, 0]),
              track_state_lens=torch.tensor([32, 0]))
    out = kp.kda_chunk_torch(**kw)
    _save("chunk_raw_tracked", **_raw_arrays(t), pool_in=_f32(pool_in), pool_out=_f32(pool),
          indices=np.array(slots), cu_seqlens=np.array(cu), track_indices=np.array([3, 0]),
          track_lens=np.array([32, 0]), lower_bound=np.float32(-5.0),
          scale=np.float32(D ** -0.5), out=_f32(out.float()))


def chunk_test_cases(tc):
    """The reference chunk test's own _reference on five of its CASES (D=64)."""
    wanted = {"ragged varlen", "zero slot", "track at 0", "track mid-chunk", "track at end"}
    for label, heads, cu, slots, track in tc.CASES:
        if label not in wanted:
            continue
        # One head keeps the fixture small; the reference draws per head alike.
        case = tc._case(1, cu, slots, track, seed=len(label))
        pool_in = case["state"].float().clone()
        ref_case = dict(case, state=tc._clone_state(case["state"]))
        out = tc._reference(ref_case)
        arr = dict(q=_bf16_bits(case["q"]), k=_bf16_bits(case["k"]), v=_bf16_bits(case["v"]),
                   a=_bf16_bits(case["a"]), b=_bf16_bits(case["b"]),
                   A_log=_f32(case["A_log"]), dt_bias=_f32(case["dt_bias"]),
                   pool_in=_f32(pool_in), pool_out=_f32(ref_case["state"]),
                   indices=np.array(slots), cu_seqlens=np.array(cu),
                   lower_bound=np.float32(tc.LOWER_BOUND), scale=np.float32(tc.SCALE),
                   out=_f32(out))
        if track is not None:
            arr["track_indices"] = np.array(track[0])
            arr["track_lens"] = np.array(track[1])
        _save("chunktest_" + label.replace(" ", "_").replace("-", "_"), **arr)


def prepared_triton(bp):
    """Triton _prepared_recurrent (interpreter), H=4, D=64, tracked."""
    import triton
    H, D, BV, T = 4, 64, 16, 33
    torch.manual_seed(99)
    qn = torch.randn(1, T, H, D) * 0.1
    kn = torch.randn(1, T, H, D) * 0.1
    v = (torch.randn(1, T, H, D) * 0.1).bfloat16()
    gdecay = torch.sigmoid(torch.randn(1, T, H, D))
    beta = torch.sigmoid(torch.randn(1, T, H))
    out = torch.zeros(1, T, H, D, dtype=torch.bfloat16)
    state = torch.randn(3, H, D, D) * 0.1           # [K,V]-contiguous, as v1 takes
    state_in = state.clone()
    indices = torch.tensor([1], dtype=torch.int32)
    starts = torch.tensor([0, T], dtype=torch.int32)
    tidx = torch.tensor([2], dtype=torch.int32)
    tlen = torch.tensor([10], dtype=torch.int32)
    bp._prepared_recurrent[(triton.cdiv(D, BV), 1, H)](
        qn, kn, v, gdecay, beta, out, state, indices, starts, tidx, tlen,
        True, H, D, BV, *state.stride(), HEAD_OFFSET=0, num_warps=1)
    _save("prepared_triton", qn=_f32(qn), kn=_f32(kn), v=_bf16_bits(v), gdecay=_f32(gdecay),
          beta=_f32(beta), state_in=_f32(state_in), state_out=_f32(state),
          indices=np.array([1]), starts=np.array([0, T]), track_indices=np.array([2]),
          track_lens=np.array([10]), out=_bf16_bits(out))


def main():
    kp, tc, bp = _load_reference()
    cfg1(kp)
    recur_raw_tracked(kp, 64, 2, 50, "recur_raw_tracked_d64", 21)
    recur_raw_tracked(kp, 128, 1, 24, "recur_raw_tracked_d128", 22)
    recur_raw_varlen(kp)
    recur_raw_varlen_intermediate(kp)
    chunk_raw(kp)
    chunk_test_cases(tc)
    prepared_triton(bp)


if __name__ == "__main__":
    main()
