#!/usr/bin/env python
"""Benchmark of the B200 GLM KDA operator (the driver's contract).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

For N > 1 launch under torchrun (one process per GPU, NCCL). Prints ONE JSON
line on rank 0.

Headline (BASELINE.json ``configs[1]``): recurrent decode, 256 requests x 1
token, H=32, K=V=128, fp32 pool of 512 slots with 256 distinct slots updated in
place; the metric is tokens/s. A step is one call of the public op
``kda_varlen_recurrent_g`` over that batch. Per-GPU work is fixed (weak
scaling): every rank owns its own 256 requests and its own pool, with no
collective on the data path; ``value`` = tokens of all ranks / max-over-ranks
device time. The touched state (512 MiB read + 512 MiB written per step) is
larger than the 126 MB L2, so no flush is needed between steps.

Also reported:
* ``roofline``: the decode kernel alone (C-ABI launches timed with CUDA events
  on the launching stream) against the measured HBM copy bandwidth;
* ``e2e``: the same metric through the public op with every step's inputs
  copied from pinned host memory and its output read back, pipelined as a
  serving loop runs it (``time_e2e``: the next step's inputs copy on a second
  stream while this step computes);
* ``cpu_baseline``: the CPU oracle (``oracle/kda_ref.py``, a port of the
  reference's PyTorch recurrence) on this host's cores, on a bounded sample;
* ``prefill``: the chunked prefill of ``configs[2]`` (8 varlen sequences,
  33,494 tokens, H=32) with its tensor/HBM roofline;
* ``prefill_long``: ``configs[3]`` (one 131,072-token sequence, 4 heads per
  GPU) through the same op;
* ``clocks``: SM clock and throttle reasons sampled by NVML during timing.

``--impl reference`` times the reference's own CPU algorithm (the oracle port;
the reference is Python and Ascend-only, so nothing of it can run on the GPU
box) on the same metric and configuration.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
for _p in (str(ROOT), str(ROOT / "01-glm53-ascend_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0

# Algorithmic bytes per (token, head) of the log-gate decode at K=V=128:
# state 64 KiB read + 64 KiB write, q/k/v bf16 768 B, g fp32 512 B, beta 4 B,
# output bf16 256 B.
DECODE_BYTES_PER_TOKEN_HEAD = 65536 * 2 + 768 + 512 + 4 + 256

# DRAM bytes (read + write) per launch from one ncu capture of each kernel:
# decode at the benchmark shape; chunk prefill captured with 8 of config 3's
# 32 heads (412,781,824 B) and scaled by 4, traffic being proportional to the
# heads processed.
DECODE_TRAFFIC_PER_LAUNCH = 1025897216
PREFILL_TRAFFIC_PER_LAUNCH = 1651127296

METRIC = "KDA tokens/s (prefill, decode) H32 d128 @1/2/4/8 B200; decode HBM GB/s vs peak"


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 0) or 0), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, FALLBACK_BF16_TFLOPS, "fallback"


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------

class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None

    def init_gpu(self):
        torch.cuda.set_device(self.local)
        if self.world > 1:
            # Keep stdout to the one JSON line: NCCL prints its version banner
            # at init unless its log level is WARN or quieter.
            if os.environ.get("NCCL_DEBUG", "").upper() in ("", "VERSION"):
                os.environ["NCCL_DEBUG"] = "WARN"
            import torch.distributed as dist
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg is not None:
            self.pg.barrier(device_ids=[self.local])
        torch.cuda.synchronize()

    def max(self, x: float) -> float:
        if self.pg is None:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ---------------------------------------------------------------------------

_REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
            0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting",
            0x10: "sync_boost", 0x100: "display_clock_setting"}


class ClockSampler(threading.Thread):
    def __init__(self, device: int, period: float = 0.02):
        super().__init__(daemon=True)
        self.period = period
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop_evt = threading.Event()
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            try:
                self.h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception as exc:  # no NVML: report what we could not sample
            self.err = f"{type(exc).__name__}: {exc}"

    def run(self):
        while self.ok and not self._stop_evt.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                self.reasons |= self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(self.period)

    def stop(self) -> dict:
        self._stop_evt.set()
        if self.is_alive():
            self.join(timeout=2)
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0,
                    "note": getattr(self, "err", "no samples")}
        names = [n for bit, n in sorted(_REASONS.items()) if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz, "reasons": names,
                "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# Timing helpers
# ---------------------------------------------------------------------------

def time_steps(fn, steps: int, warmup: int, dist: Dist, stream=None):
    """W untimed steps, then exactly K timed steps bracketed by barrier+sync;
    returns the max-over-ranks device milliseconds of the K steps."""
    for _ in range(warmup):
        fn()
    dist.barrier()
    s = stream or torch.cuda.current_stream()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s)
    for _ in range(steps):
        fn()
    end.record(s)
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(start.elapsed_time(end))


def time_e2e(host: dict, run, out_shape, steps: int, warmup: int, dist: Dist):
    """Per-step device milliseconds of the op end to end from pinned host
    buffers, pipelined as a serving loop runs it: while step i computes on the
    current stream, step i+1's inputs copy host->device on two copy streams
    (the inputs split between them by size, so two copy engines share the
    link; two device input sets, each reused only after the op that read it is
    done), and step i's bf16 output is read back into pinned host memory on a
    further stream. The timed region holds exactly `steps` input copies and `steps`
    read-backs: it opens before the copy for the first timed step's successor
    and closes after the last copy and the last read-back have finished.
    Returns (ms per step, host->device bytes per step, device->host bytes per
    step)."""
    cs = torch.cuda.current_stream()
    xss, ds = (torch.cuda.Stream(), torch.cuda.Stream()), torch.cuda.Stream()
    devs = [{n: torch.empty_like(t, device="cuda") for n, t in host.items()} for _ in range(2)]
    out_host = [torch.empty(out_shape, dtype=torch.bfloat16).pin_memory() for _ in range(2)]
    # inputs -> copy stream, largest first onto the less loaded one
    groups, load = ([], []), [0, 0]
    for n, t in sorted(host.items(), key=lambda kv: -kv[1].numel() * kv[1].element_size()):
        g = 0 if load[0] <= load[1] else 1
        groups[g].append(n)
        load[g] += t.numel() * t.element_size()
    copied = [[torch.cuda.Event(), torch.cuda.Event()] for _ in range(2)]   # [set][stream]
    used = [torch.cuda.Event(), torch.cuda.Event()]
    read = torch.cuda.Event()
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    d2h = out_host[0].numel() * out_host[0].element_size()
    it = [0]

    def copy_in(b):
        for k, xs in enumerate(xss):
            xs.wait_event(used[b])             # the op that last read set b has finished
            with torch.cuda.stream(xs):
                for n in groups[k]:
                    devs[b][n].copy_(host[n], non_blocking=True)
            copied[b][k].record(xs)

    def wait_copied(b):
        for ev in copied[b]:
            cs.wait_event(ev)

    def e2e_step():
        b = it[0] & 1
        copy_in(b ^ 1)                         # inputs of the next step
        wait_copied(b)
        o = run(devs[b])
        used[b].record(cs)
        ds.wait_stream(cs)
        with torch.cuda.stream(ds):
            out_host[b].copy_(o, non_blocking=True)
        o.record_stream(ds)
        read.record(ds)
        it[0] += 1

    copy_in(0)
    for _ in range(warmup):
        e2e_step()
    torch.cuda.synchronize()
    dist.barrier()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(cs)
    for xs in xss:
        xs.wait_event(start)                   # no timed copy starts before the region opens
    # The first timed step's own inputs were copied during the last warm-up
    # step; its successor's copy is the first of the `steps` timed copies.
    wait_copied(it[0] & 1)
    for _ in range(steps):
        e2e_step()
    wait_copied(it[0] & 1)                     # the last timed copy
    cs.wait_event(read)                        # the last read-back
    end.record(cs)
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(start.elapsed_time(end)) / steps, h2d, d2h


# ---------------------------------------------------------------------------
# Decode (headline)
# ---------------------------------------------------------------------------

def bench_decode(args, dist: Dist, hbm_gbs: float, peak_kind: str) -> dict:
    from sgl_glm53_ascend_ops import abi, ops, workloads

    w = workloads.config2(seed=1000 + dist.rank)
    d = w.to("cuda")
    kw = d.kwargs()
    tokens = w.tokens
    heads = w.heads

    def step():
        ops.kda_varlen_recurrent_g(**kw, prefill=False)

    sampler = ClockSampler(dist.local)
    sampler.start()
    ms = time_steps(step, args.steps, args.warmup, dist)
    clocks = sampler.stop()
    ms_per_step = ms / args.steps
    value = dist.world * tokens / (ms_per_step / 1e3)

    # Kernel alone through the C ABI (same stream, CUDA events).
    out = torch.empty_like(d.v)
    cargs = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=d.pool, indices=d.indices,
                                  cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                  g=d.g, beta=d.beta)

    def launch():
        rc = abi.recurrent_launch(cargs)
        if rc != 0:
            raise RuntimeError(f"kda_recurrent_launch: {abi.status_string(rc)}")

    kms = time_steps(launch, args.steps, args.warmup, dist) / args.steps
    alg_bytes = tokens * heads * DECODE_BYTES_PER_TOKEN_HEAD
    achieved = alg_bytes / (kms / 1e3) / 1e9
    roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_gbs, "unit": "GB/s",
                "frac": round(achieved / hbm_gbs, 4), "traffic": DECODE_TRAFFIC_PER_LAUNCH,
                "kernel_us": round(kms * 1e3, 2), "algorithmic_bytes": alg_bytes,
                "peak_source": f"{peak_kind} hbm_gbs (MEASURED_PEAKS.json)" if peak_kind == "measured"
                else "fallback 6.65 TB/s"}

    # End to end through the public op from pinned host buffers.
    host = {n: t.cpu().pin_memory() for n, t in
            dict(q=w.q, k=w.k, v=w.v, g=w.g, beta=w.beta, indices=w.indices, cu=w.cu_seqlens).items()}

    def run(dev):
        return ops.kda_varlen_recurrent_g(q=dev["q"], k=dev["k"], v=dev["v"], g=dev["g"], beta=dev["beta"],
                                          initial_state_source=d.pool, initial_state_indices=dev["indices"],
                                          cu_seqlens=dev["cu"], scale=d.scale, prefill=False)

    ems, h2d, d2h = time_e2e(host, run, w.v.shape, args.steps, args.warmup, dist)
    e2e = {"value": round(dist.world * tokens / (ems / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ems, 4),
           "pipelining": "step i+1's inputs copy host->device on two copy streams while step i runs "
                         "(two device input sets); each step's output is read back on a further stream"}
    return dict(value=value, ms_per_step=ms_per_step, roofline=roofline, e2e=e2e, clocks=clocks,
                gpu_launches=args.steps, tokens=tokens)


# ---------------------------------------------------------------------------
# Chunked prefill
# ---------------------------------------------------------------------------

# Dense tensor-core work per (token, head) of the chunk-64 algorithm at
# K=V=128 (A_kk, A_qk, W, U, W.S, Q.S, Aqk.V', state update; the triangular
# solve excluded) and the minimal HBM bytes per (token, head): q/k/v bf16,
# g fp32, beta, output bf16.
PREFILL_FLOPS_PER_TOKEN_HEAD = 180224
PREFILL_BYTES_PER_TOKEN_HEAD = 768 + 512 + 4 + 256


def bench_prefill(args, dist: Dist, hbm_gbs: float, bf16_tf: float, steps: int, warmup: int) -> dict:
    from sgl_glm53_ascend_ops import abi, ops, workloads

    w = workloads.config3(seed=2000 + dist.rank)
    d = w.to("cuda")
    kw = d.kwargs()
    tokens, heads = w.tokens, w.heads

    def step():
        ops.kda_varlen_chunk_g(**kw, prefill=True)

    ms = time_steps(step, steps, warmup, dist) / steps
    # The chunk kernel alone through the C ABI (the workspace is allocated once).
    out = torch.empty_like(d.v)
    cargs = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=d.pool, indices=d.indices,
                                  cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                  g=d.g, beta=d.beta)
    nws = abi.chunk_workspace_bytes(w.indices.numel(), tokens, heads, w.dim)
    ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")

    def launch():
        rc = abi.chunk_launch(cargs, ws, nws)
        if rc != 0:
            raise RuntimeError(f"kda_chunk_launch: {abi.status_string(rc)}")

    kms = time_steps(launch, steps, warmup, dist) / steps
    flops = tokens * heads * PREFILL_FLOPS_PER_TOKEN_HEAD
    min_bytes = tokens * heads * PREFILL_BYTES_PER_TOKEN_HEAD + 2 * len(w.lengths) * heads * 65536
    tflops = flops / (kms / 1e3) / 1e12
    floor_ms = max(flops / (bf16_tf * 1e12), min_bytes / (hbm_gbs * 1e9)) * 1e3
    return {
        "metric": "KDA prefill tokens/s (chunk-64, configs[2])",
        "value": round(dist.world * tokens / (ms / 1e3), 1),
        "unit": "tokens/s",
        "ms_per_step": round(ms, 4),
        "steps": steps,
        "warmup": warmup,
        "config": {"workload": f"cfg3: 8 varlen sequences {w.lengths} (total {tokens}), H=32, K=V=128, "
                               "zero initial state, log-gate op",
                   "l2": "inputs larger than L2 (1.4 GB per step), no flush"},
        "roofline": {"bound": "hbm", "achieved": round(min_bytes / (kms / 1e3) / 1e9, 1), "peak": hbm_gbs,
                     "unit": "GB/s", "frac": round(min_bytes / (kms / 1e3) / 1e9 / hbm_gbs, 4),
                     "traffic": PREFILL_TRAFFIC_PER_LAUNCH, "kernel_us": round(kms * 1e3, 1),
                     "algorithmic_bytes": min_bytes,
                     "tensor_tflops": round(tflops, 1), "tensor_frac": round(tflops / bf16_tf, 4),
                     "attainable_frac": round(floor_ms / kms, 4),
                     "note": "algorithmic FLOPs 180,224/token-head (bf16x3 split issues 3x that on the "
                             "tensor pipe); attainable = max(flop floor, byte floor) / time"},
        "gpu_launches": 2 * steps,
    }


def bench_prefill_long(args, dist: Dist, steps: int, warmup: int) -> dict:
    """one 131,072-token sequence, 4 heads per GPU (the
    configuration shards H=32 as 4 heads on each of 8 GPUs), fp32 initial
    state from the pool. Every chunk of a head follows the previous one, so
    this measures the serial inter-chunk state pass."""
    from sgl_glm53_ascend_ops import ops, workloads

    heads = 4
    w = workloads.config4(seed=3000 + dist.rank, heads=heads)
    d = w.to("cuda")
    kw = d.kwargs()
    pool0 = d.pool.clone()

    def step():
        ops.kda_varlen_chunk_g(**kw, prefill=True)

    ms = time_steps(step, steps, warmup, dist) / steps
    d.pool.copy_(pool0)

    # The inter-chunk state pass on its own: the same launch through the C
    # ABI's measurement hook, CUDA events between the split path's kernels.
    from sgl_glm53_ascend_ops import abi
    out = torch.empty_like(d.v)
    cargs = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=out, state=d.pool, indices=d.indices,
                                  cu_seqlens=d.cu_seqlens, scale=d.scale, gate_mode=abi.KDA_GATE_LOG,
                                  g=d.g, beta=d.beta)
    nws = abi.chunk_workspace_bytes(1, w.tokens, heads, 128)
    ws = torch.empty(nws, dtype=torch.uint8, device="cuda")
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(6)] for _ in range(steps)]
    for e in (x for row in evs for x in row):
        e.record()                                  # creates the event handles
    torch.cuda.synchronize()
    for i in range(steps):
        rc = abi.chunk_launch_phases(cargs, ws, nws, evs[i])
        if rc != 0:
            raise RuntimeError(f"kda_chunk_launch_phases: {abi.status_string(rc)}")
    torch.cuda.synchronize()
    d.pool.copy_(pool0)
    names = ("plan_prep", "scan_first_pass", "combine", "rescan", "outputs")
    phases = {n: round(dist.max(sum(evs[i][j].elapsed_time(evs[i][j + 1]) for i in range(steps)) / steps), 4)
              for j, n in enumerate(names)}
    del ws
    return {
        "metric": "KDA long-context prefill tokens/s (chunk-64, configs[3])",
        "value": round(dist.world * w.tokens * heads / (ms / 1e3), 1),
        "unit": "token-heads/s",
        "ms_per_step": round(ms, 4),
        "per_chunk_us": round(ms * 1e3 / (w.tokens / 64), 3),
        "state_pass_ms": round(phases["scan_first_pass"] + phases["combine"] + phases["rescan"], 4),
        "phases_ms": phases,
        "steps": steps,
        "warmup": warmup,
        "config": {"workload": f"cfg4: 1 sequence x {w.tokens} tokens, {heads} heads per GPU (of H=32), "
                               "K=V=128, fp32 initial state ~ 0.1 N(0,1), log-gate op",
                   "scaling": "weak (4 heads per GPU)"},
    }


def cpu_prefill_rate(tokens: int, budget_s: float, seed: int = 8):
    """tokens/s of the CPU chunk oracle on one sequence of `tokens` tokens, H=32."""
    from oracle import kda_ref
    from sgl_glm53_ascend_ops import workloads

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = workloads.config3(seed=seed, lengths=[tokens])
    reps, t0 = 0, time.perf_counter()
    while True:
        kda_ref.kda_varlen_chunk_g(**w.kwargs(), out_fp32=True)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return reps * tokens / el, threads, f"{reps} x one {tokens}-token sequence x 32 heads (chunk oracle), {el:.1f} s"


# ---------------------------------------------------------------------------
# CPU baseline (rank 0, N = 1): the oracle port on this host's cores
# ---------------------------------------------------------------------------

def cpu_decode_rate(requests: int, budget_s: float, seed: int = 7):
    """tokens/s of the CPU oracle on `requests` cfg2-shaped requests; repeats
    until `budget_s` seconds of work. Returns (rate, threads, sample text)."""
    from oracle import kda_ref
    from sgl_glm53_ascend_ops import workloads

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    w = workloads.config2(seed=seed, requests=requests, slots=requests + 1)
    reps, t0 = 0, time.perf_counter()
    while True:
        kda_ref.kda_varlen_recurrent_g(**w.kwargs(), out_fp32=True)
        reps += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    return reps * w.tokens / el, threads, f"{reps} x {requests} decode requests x 32 heads, {el:.1f} s"


def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return
    from oracle import kda_ref
    from sgl_glm53_ascend_ops import workloads

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    sample_req = 8
    w = workloads.config2(seed=11, requests=sample_req, slots=sample_req + 1)

    def step():
        kda_ref.kda_varlen_recurrent_g(**w.kwargs(), out_fp32=True)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = args.steps * w.tokens / el
    sample = f"each step: {sample_req} of config 2's 256 requests x 32 heads (oracle port, fp32)"
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg2 decode: 256 req x 1 tok, H=32, K=V=128, pool 512 slots (sampled)",
                       "parallelism": "host cores"},
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU-oracle work")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--mode", choices=("full", "kernel", "prefill-kernel", "prefill-long"), default="full",
                    help="kernel / prefill-kernel: only the timed decode / chunk op loop (profiler captures)")
    ap.add_argument("--prefill-heads", type=int, default=32,
                    help="prefill-kernel mode: heads of config 3 (fewer keeps a full ncu capture small)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return

    dist.init_gpu()
    hbm_gbs, bf16_tf, bf16_tf_sus, peak_kind = _peaks()
    if args.mode == "prefill-kernel":
        from sgl_glm53_ascend_ops import ops, workloads
        kw = workloads.config3(seed=2000 + dist.rank, heads=args.prefill_heads).to("cuda").kwargs()
        ms = time_steps(lambda: ops.kda_varlen_chunk_g(**kw, prefill=True), args.steps, args.warmup, dist)
        if dist.rank == 0:
            print(json.dumps({"mode": "prefill-kernel", "ms_per_step": ms / args.steps}), flush=True)
        dist.close()
        return
    if args.mode == "prefill-long":
        r = bench_prefill_long(args, dist, steps=args.steps, warmup=args.warmup)
        if dist.rank == 0:
            print(json.dumps({"mode": "prefill-long", **r}), flush=True)
        dist.close()
        return
    if args.mode == "kernel":
        from sgl_glm53_ascend_ops import ops, workloads
        kw = workloads.config2(seed=1000 + dist.rank).to("cuda").kwargs()
        ms = time_steps(lambda: ops.kda_varlen_recurrent_g(**kw, prefill=False), args.steps, args.warmup, dist)
        if dist.rank == 0:
            print(json.dumps({"mode": "kernel", "ms_per_step": ms / args.steps}), flush=True)
        dist.close()
        return
    dec = bench_decode(args, dist, hbm_gbs, peak_kind)

    pre = bench_prefill(args, dist, hbm_gbs, bf16_tf, steps=args.prefill_steps, warmup=3)
    pre_long = bench_prefill_long(args, dist, steps=20, warmup=3)

    cpu = None
    if dist.rank == 0 and dist.world == 1:
        rate, threads, sample = cpu_decode_rate(32, args.cpu_budget)
        cpu = {"value": round(rate, 2), "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}
        prate, pthreads, psample = cpu_prefill_rate(512, args.cpu_budget)
        pre["cpu_baseline"] = {"value": round(prate, 2), "unit": "tokens/s", "cores": pthreads, "kind": "port",
                               "sample": psample}

    if dist.rank == 0:
        line = {
            "metric": METRIC,
            "value": round(dec["value"], 1),
            "unit": "tokens/s",
            "n_gpus": dist.world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(dec["ms_per_step"], 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "cfg2 decode: 256 req x 1 tok, H=32, K=V=128, fp32 pool 512 slots, "
                                   "256 distinct slots updated in place (log-gate op)",
                       "global_batch": 256 * dist.world, "per_gpu_batch": 256,
                       "l2": "inputs larger than L2 (1 GiB of state traffic per step), no flush",
                       "parallelism": f"dp{dist.world} (independent request batches, no collective)"},
            "roofline": dec["roofline"],
            "cpu_baseline": cpu,
            "e2e": dec["e2e"],
            "gpu_launches": dec["gpu_launches"],
            "clocks": dec["clocks"],
            "prefill": pre,
            "prefill_long": pre_long,
        }
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
