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
  33,494 tokens, H=32) with its tensor/HBM roofline, per rank (weak);
* ``prefill_strong`` / ``mixed``: ``configs[2]`` and ``configs[4]`` (64
  one-token requests + 4 resumed 2048-token prefills) split 32/N heads per
  rank (strong scaling), verified after timing against one GPU running all
  heads (outputs and updated slots gathered with NCCL on rank 0, untouched
  slots checked on every rank);
* ``prefill_long``: ``configs[3]`` (one 131,072-token sequence, 4 heads per
  GPU) through the same op, with the split path's phases and DRAM traffic;
* ``published_shapes``: every shape the reference publishes an Ascend 910B
  time for (decode H16/32/64 x B1/32/128, the five verify shapes with the
  commit, chunk prefill H8 x T1024/2048/4096), through the raw-gate ops;
* ``frontend``: the causal-conv front end that feeds the op (``kda_causal_conv1d``)
  on config 3's prefill and config 2's decode shapes at H=32, against HBM;
* ``clocks``: SM clock and throttle reasons sampled by NVML during timing.

``--lines`` picks the secondary lines (default: all). ``--impl reference``
times the reference's own CPU algorithm (the oracle port; the reference is
PyTorch plus Ascend-only kernels, so nothing of it can run on the GPU box) on
the headline's exact workload, loading no library of this repository.
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
# configs[3] (4 heads), all six kernels of one split-path call (plan, prep,
# scan, combine, rescan, outputs): captured at 32,768 tokens (1,318,200,832 B)
# and scaled by 4, the traffic being proportional to the chunks processed.
PREFILL_LONG_TRAFFIC_PER_LAUNCH = 5272803328

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

    def all_true(self, ok: bool) -> bool:
        if self.pg is None:
            return ok
        t = torch.tensor([0.0 if ok else 1.0], dtype=torch.float64, device="cuda")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item()) == 0.0

    def gather_heads(self, x: torch.Tensor, dim: int) -> torch.Tensor:
        """One NCCL all-gather of every rank's head shard `x` (same shape on all
        ranks), reassembled along the head dimension `dim` in rank order."""
        if self.pg is None:
            return x
        x = x.contiguous()
        buf = torch.empty(self.world * x.numel(), dtype=x.dtype, device=x.device)
        self.pg.all_gather_into_tensor(buf, x.reshape(-1))
        return torch.cat(list(buf.view((self.world,) + tuple(x.shape)).unbind(0)), dim=dim)

    def close(self):
        if self.pg is not None:
            self.pg.destroy_process_group()


def bind_local_cpus(device: int):
    """Pins this process to the CPUs NVML reports as local to `device` (its
    NUMA node), as a serving process is pinned, so the pinned host buffers of
    the end-to-end line are allocated and first touched on the GPU's own node.
    Returns (previous CPU set, local CPU list), or None when NVML cannot say."""
    try:
        import pynvml
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        try:
            h = pynvml.nvmlDeviceGetHandleByUUID(uuid if uuid.startswith("GPU-") else "GPU-" + uuid)
        except Exception:
            h = pynvml.nvmlDeviceGetHandleByIndex(device)
        words = pynvml.nvmlDeviceGetCpuAffinity(h, 16)
        local = [64 * i + b for i, w in enumerate(words) for b in range(64) if (int(w) >> b) & 1]
        prev = os.sched_getaffinity(0)
        local = sorted(set(local) & prev)
        if not local:
            return None
        os.sched_setaffinity(0, local)
        return prev, local
    except Exception:
        return None


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


_FLUSH = None


def time_flushed(fn, iters: int, warmup: int, dist: Dist):
    """Per-call device milliseconds of a small workload that fits in L2: before
    every call a 256 MiB buffer (twice the 126 MB L2) is rewritten, so the call
    reads its inputs from HBM; CUDA events bracket the call alone, on the
    launching stream. Returns the max over ranks of the per-rank median."""
    global _FLUSH
    if _FLUSH is None:
        _FLUSH = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    for _ in range(warmup):
        fn()
    dist.barrier()
    s = torch.cuda.current_stream()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        _FLUSH.fill_(1)
        # Keep the GPU busy while the host enqueues the call, so the interval
        # holds device time only (no host launch latency).
        torch.cuda._sleep(200_000)
        a.record(s)
        fn()
        b.record(s)
    torch.cuda.synchronize()
    dist.barrier()
    return dist.max(statistics.median(a.elapsed_time(b) for a, b in ev))


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


def h2d_link_gbs(host: dict, reps: int) -> float:
    """Host->device copy rate of the end-to-end line's own pinned buffers
    (same two copy streams, nothing else running): the link bound that the
    end-to-end number is read against."""
    xss = (torch.cuda.Stream(), torch.cuda.Stream())
    dev = {n: torch.empty_like(t, device="cuda") for n, t in host.items()}
    names = sorted(host, key=lambda n: -host[n].numel() * host[n].element_size())
    groups, load = ([], []), [0, 0]
    for n in names:
        g = 0 if load[0] <= load[1] else 1
        groups[g].append(n)
        load[g] += host[n].numel() * host[n].element_size()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cs = torch.cuda.current_stream()
    start.record(cs)
    for xs in xss:
        xs.wait_event(start)
    for _ in range(reps):
        for k, xs in enumerate(xss):
            with torch.cuda.stream(xs):
                for n in groups[k]:
                    dev[n].copy_(host[n], non_blocking=True)
    for xs in xss:
        cs.wait_stream(xs)
    end.record(cs)
    torch.cuda.synchronize()
    nbytes = reps * sum(t.numel() * t.element_size() for t in host.values())
    return nbytes / (start.elapsed_time(end) / 1e3) / 1e9


# ---------------------------------------------------------------------------
# Decode (headline)
# ---------------------------------------------------------------------------

def bench_decode(args, dist: Dist, hbm_gbs: float, peak_kind: str) -> dict:
    import kda_workloads as workloads
    from sgl_glm53_ascend_ops import abi, ops

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
    link = h2d_link_gbs(host, max(args.steps, 20))
    e2e = {"value": round(dist.world * tokens / (ems / 1e3), 1), "unit": "tokens/s",
           "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ems, 4),
           "h2d_link_gbs": round(link, 1), "h2d_frac_of_link": round(h2d / (ems / 1e3) / 1e9 / link, 4),
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
    import kda_workloads as workloads
    from sgl_glm53_ascend_ops import abi, ops

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
    import kda_workloads as workloads
    from sgl_glm53_ascend_ops import ops

    heads = 4
    w = workloads.config4(seed=3000 + dist.rank, heads=heads, tokens=getattr(args, "long_tokens", 131072))
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
    hbm_gbs, bf16_tf = args.peaks[0], args.peaks[1]
    flops = w.tokens * heads * PREFILL_FLOPS_PER_TOKEN_HEAD
    min_bytes = w.tokens * heads * PREFILL_BYTES_PER_TOKEN_HEAD + 2 * heads * 65536
    floor_ms = max(flops / (bf16_tf * 1e12), min_bytes / (hbm_gbs * 1e9)) * 1e3
    gbs = min_bytes / (ms / 1e3) / 1e9
    tflops = flops / (ms / 1e3) / 1e12
    return {
        "metric": "KDA long-context prefill tokens/s (chunk-64, configs[3])",
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_gbs, "unit": "GB/s",
                     "frac": round(gbs / hbm_gbs, 4), "traffic": PREFILL_LONG_TRAFFIC_PER_LAUNCH,
                     "algorithmic_bytes": min_bytes, "algorithmic_flops": flops,
                     "tensor_tflops": round(tflops, 1), "tensor_frac": round(tflops / bf16_tf, 4),
                     "attainable_frac": round(floor_ms / ms, 4),
                     "note": "one call of the op (plan, prep, scan, combine, rescan, outputs); traffic = DRAM "
                             "bytes of all its kernels per call"},
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


# ---------------------------------------------------------------------------
# Head-sharded lines (BASELINE configs[2] strong-scaled, configs[4] mixed)
# ---------------------------------------------------------------------------

def _bf16_out_err(got: torch.Tensor, ref: torch.Tensor) -> float:
    """max |got - ref| / rms(ref) with one bf16 ulp of ref credited (both
    sides are bf16 outputs of the operator)."""
    got, ref = got.float(), ref.float()
    rms = ref.pow(2).mean().sqrt().clamp_min(1e-30)
    _, e = torch.frexp(ref)
    credit = torch.ldexp(torch.ones_like(ref), e - 8)
    return float(((got - ref).abs() - credit).clamp_min(0).max() / rms)


def bench_head_sharded(w, steps: int, warmup: int, dist: Dist, hbm_gbs: float, bf16_tf: float) -> dict:
    """The global workload `w` (all H heads) split H/N heads per rank, as
    tensor parallelism by heads places it: rank r owns heads [r H/N, (r+1) H/N)
    of the token tensors and that slice of the state pool. A step is one call
    of the chunk op (`kda_varlen_chunk_g`) on every rank; value = the global
    workload's tokens / the max-over-ranks device time, so the total work is
    the same at every N (strong scaling).

    Verification, outside the timed region: every rank reruns its shard from
    the initial pool and checks that the slots no request names are
    bit-identical; the shards' outputs and updated slots are assembled on rank
    0 with one NCCL all-gather each and compared with one GPU running all H
    heads in a single call."""
    from sgl_glm53_ascend_ops import ops

    N, H = dist.world, w.heads
    sh = w.head_shard(dist.rank, N) if N > 1 else w
    d = sh.to("cuda")
    pool0 = d.pool.clone()
    kw = d.kwargs()

    def step():
        ops.kda_varlen_chunk_g(**kw, prefill=True)

    ms = time_steps(step, steps, warmup, dist) / steps

    d.pool.copy_(pool0)
    out = ops.kda_varlen_chunk_g(**kw, prefill=True)
    touched = sorted({int(x) for x in w.indices.tolist()} - {0})
    tidx = torch.tensor(touched, dtype=torch.long, device="cuda")
    other = torch.ones(d.pool.shape[0], dtype=torch.bool, device="cuda")
    other[tidx] = False
    untouched_ok = dist.all_true(bool(torch.equal(d.pool[other], pool0[other])))
    out_all = dist.gather_heads(out, dim=2)
    st_all = dist.gather_heads(d.pool[tidx], dim=1)
    del d, pool0, out, kw
    verify = {"untouched_slots_bit_equal": untouched_ok, "assembled": "NCCL all_gather on rank 0, outside timing"}
    if dist.rank == 0:
        full = w.to("cuda")
        ref = ops.kda_varlen_chunk_g(**full.kwargs(), prefill=True)
        ref_st = full.pool[tidx]
        oe = _bf16_out_err(out_all, ref)
        se = float((st_all - ref_st).norm() / ref_st.norm().clamp_min(1e-30))
        verify.update({"vs_one_gpu_all_heads": {"bit_equal": bool(torch.equal(out_all, ref) and
                                                                   torch.equal(st_all, ref_st)),
                                                "out_err": oe, "state_err": se},
                       "ok": bool(untouched_ok and oe <= 5e-3 and se <= 1e-3)})
        del full, ref, ref_st
    del out_all, st_all
    torch.cuda.empty_cache()

    tokens, reqs = w.tokens, len(w.lengths)
    flops = tokens * H * PREFILL_FLOPS_PER_TOKEN_HEAD
    min_bytes = tokens * H * PREFILL_BYTES_PER_TOKEN_HEAD + 2 * reqs * H * 65536
    gpu_s = N * ms / 1e3                          # GPU-seconds per step, all ranks
    tflops = flops / gpu_s / 1e12
    gbs = min_bytes / gpu_s / 1e9
    floor_s = max(flops / (bf16_tf * 1e12), min_bytes / (hbm_gbs * 1e9))
    return {
        "value": round(tokens / (ms / 1e3), 1),
        "unit": "tokens/s",
        "ms_per_step": round(ms, 4),
        "steps": steps,
        "warmup": warmup,
        "n_gpus": N,
        "heads_per_gpu": H // N,
        "scaling": "strong",
        "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": hbm_gbs, "unit": "GB/s",
                     "frac": round(gbs / hbm_gbs, 4), "tensor_tflops": round(tflops, 1),
                     "tensor_frac": round(tflops / bf16_tf, 4), "attainable_frac": round(floor_s * N / gpu_s, 4),
                     "algorithmic_bytes": min_bytes, "algorithmic_flops": flops,
                     "note": "per-GPU average: global work / (N x max-over-ranks time)"},
        "verify": verify,
    }


def bench_prefill_strong(args, dist: Dist, hbm_gbs: float, bf16_tf: float, steps: int, warmup: int) -> dict:
    import kda_workloads as workloads

    w = workloads.config3(seed=2000)
    r = bench_head_sharded(w, steps, warmup, dist, hbm_gbs, bf16_tf)
    r["metric"] = "KDA prefill tokens/s, configs[2] head-sharded (32/N heads per GPU)"
    r["config"] = {"workload": f"cfg3: 8 varlen sequences {w.lengths} (total {w.tokens}), H=32 split "
                               f"{32 // dist.world} per GPU, K=V=128, zero initial state, log-gate op",
                   "parallelism": f"tp{dist.world} by heads, no collective on the data path",
                   "l2": "inputs larger than L2 at every N (>= 170 MB per rank per step), no flush"}
    return r


def bench_mixed(args, dist: Dist, hbm_gbs: float, bf16_tf: float, steps: int, warmup: int) -> dict:
    import kda_workloads as workloads

    w = workloads.config5(seed=5000)
    r = bench_head_sharded(w, steps, warmup, dist, hbm_gbs, bf16_tf)
    r["metric"] = "KDA mixed-batch tokens/s, configs[4] head-sharded (32/N heads per GPU)"
    r["config"] = {"workload": "cfg5: 64 one-token decode requests + 4 x 2048-token prefills resumed from "
                               "nonzero pooled states (1024-slot pool, 68 distinct slots), H=32 split "
                               f"{32 // dist.world} per GPU, K=V=128, one chunk-op call, log-gate op",
                   "parallelism": f"tp{dist.world} by heads, no collective on the data path",
                   "l2": "inputs larger than L2 at every N, no flush"}
    return r


# ---------------------------------------------------------------------------
# The reference's published shapes (Ascend 910B numbers, context only)
# ---------------------------------------------------------------------------

# Raw-gate bytes per (token, head): q, k, v, a bf16 (4 x 256), b bf16, out bf16.
RAW_TOKEN_BYTES = 4 * 256 + 2 + 256

# bench/kda_recurrent/DISCARDED-cann-recurrent-kda.md:22-30 (ascendc column, ms)
PUBLISHED_DECODE_MS = {(16, 1): 0.121, (16, 32): 0.133, (16, 128): 0.303, (32, 1): 0.118, (32, 32): 0.146,
                       (32, 128): 0.633, (64, 1): 0.140, (64, 32): 0.301, (64, 128): 1.225}
# bench/kda_recurrent/bench_kda_varlen_recurrent.py:90-114 (label, heads, requests),
# 4 draft tokens per request; published at
# sgl-glm53-ascend-ops/csrc/kda/recurrent/kda_varlen_recurrent_decode.h:807-808.
VERIFY_SHAPES = (("256K DP4TP2", 32, 2), ("256K DP2TP4", 16, 3), ("256K DP8TP1", 64, 1),
                 ("512K DP4TP2", 32, 1), ("512K DP2TP4", 16, 1))
PUBLISHED_VERIFY_US = {"512K DP4TP2": 23.8, "512K DP2TP4": 19.7}
DRAFT_TOKENS = 4
# bench/kda_chunk/README.md:35-39 (H8 C64, ascendc column, ms)
PUBLISHED_CHUNK_MS = {1024: 2.03, 2048: 3.83, 4096: 7.36}


def _raw_case(heads: int, lengths, slots: int, seed: int):
    """The reference benches' inputs (bench_kda_varlen_recurrent.py make_case,
    bench_kda_chunk.py): q, k, v, a ~ 0.2 N(0,1) bf16, b ~ N(0,1) bf16, A_log and
    dt_bias ~ 0.1 N(0,1), pool ~ 0.1 N(0,1) K-contiguous, requests in slots 1..B."""
    g = torch.Generator(device="cuda").manual_seed(seed)
    T, D = sum(lengths), 128
    kw = {n: (torch.randn(1, T, heads, D, generator=g, device="cuda") * 0.2).bfloat16() for n in "qkva"}
    kw["b"] = torch.randn(1, T, heads, generator=g, device="cuda").bfloat16()
    kw["A_log"] = torch.randn(heads, generator=g, device="cuda") * 0.1
    kw["dt_bias"] = torch.randn(heads * D, generator=g, device="cuda") * 0.1
    kw["initial_state_source"] = (torch.randn(slots, heads, D, D, generator=g, device="cuda") * 0.1).transpose(-1, -2)
    kw["initial_state_indices"] = torch.arange(1, len(lengths) + 1, dtype=torch.int32, device="cuda")
    cu = [0]
    for n in lengths:
        cu.append(cu[-1] + n)
    kw["cu_seqlens"] = torch.tensor(cu, dtype=torch.int32, device="cuda")
    kw["lower_bound"] = -5.0
    kw["scale"] = D ** -0.5
    return kw


def bench_published_shapes(args, dist: Dist, hbm_gbs: float, bf16_tf: float, iters: int, warmup: int) -> dict:
    """Each shape the reference publishes an Ascend time for, through the
    reference's own raw-gate ops on one GPU (every rank runs the same shapes;
    the max over ranks is reported). Each call is timed alone with CUDA events
    after an L2 flush (the inputs fit in L2); the median of `iters` calls."""
    from sgl_glm53_ascend_ops import ops

    decode = []
    for H in (16, 32, 64):
        for B in (1, 32, 128):
            kw = _raw_case(H, [1] * B, B + 1, seed=H * 1000 + B)
            ms = time_flushed(lambda: ops.kda_varlen_recurrent(**kw, prefill=False), iters, warmup, dist)
            nbytes = B * H * (2 * 65536 + RAW_TOKEN_BYTES)
            pub = PUBLISHED_DECODE_MS[(H, B)]
            decode.append({"heads": H, "batch": B, "us": round(ms * 1e3, 2), "tokens_per_s": round(B / (ms / 1e3), 1),
                           "hbm_gbs": round(nbytes / (ms / 1e3) / 1e9, 1),
                           "hbm_frac": round(nbytes / (ms / 1e3) / 1e9 / hbm_gbs, 4),
                           "ascend_910b_ms": pub, "speedup_vs_ascend": round(pub / ms, 2)})
            del kw
    verify = []
    for label, H, R in VERIFY_SHAPES:
        kw = _raw_case(H, [DRAFT_TOKENS] * R, R + 1, seed=H * 100 + R)
        mid = (torch.randn(R, DRAFT_TOKENS, H, 128, 128, device="cuda") * 0.1).transpose(-1, -2)
        ms = time_flushed(lambda: ops.kda_varlen_recurrent(**kw, intermediate_state=mid, prefill=False),
                          iters, warmup, dist)
        # Commit: every request accepts its step 2 (dst = the pool's physical
        # [layers=1, slots, H, V, K] view, src = the checkpoints').
        dst = kw["initial_state_source"].unsqueeze(0).transpose(-1, -2)
        src = mid.unsqueeze(0).transpose(-1, -2)
        di = kw["initial_state_indices"]
        si = torch.arange(R, dtype=torch.int32, device="cuda")
        st = torch.full((R,), 2, dtype=torch.int32, device="cuda")
        cms = time_flushed(lambda: ops.move_intermediate_cache_kda(dst, src, di, si, st), iters, warmup, dist)
        vbytes = R * H * (65536 + DRAFT_TOKENS * 65536 + DRAFT_TOKENS * RAW_TOKEN_BYTES)
        cbytes = R * H * 2 * 65536
        row = {"shape": label, "heads": H, "requests": R, "draft_tokens": DRAFT_TOKENS,
               "verify_us": round(ms * 1e3, 2), "verify_hbm_gbs": round(vbytes / (ms / 1e3) / 1e9, 1),
               "verify_hbm_frac": round(vbytes / (ms / 1e3) / 1e9 / hbm_gbs, 4),
               "commit_us": round(cms * 1e3, 2), "commit_hbm_gbs": round(cbytes / (cms / 1e3) / 1e9, 1)}
        if label in PUBLISHED_VERIFY_US:
            row["ascend_910b_us"] = PUBLISHED_VERIFY_US[label]
            row["speedup_vs_ascend"] = round(PUBLISHED_VERIFY_US[label] / (ms * 1e3), 2)
        verify.append(row)
        del kw, mid
    chunk = []
    for T in (1024, 2048, 4096):
        kw = _raw_case(8, [T], 2, seed=T)
        ms = time_flushed(lambda: ops.kda_varlen_chunk(**kw, prefill=True), iters, warmup, dist)
        flops = T * 8 * PREFILL_FLOPS_PER_TOKEN_HEAD
        pub = PUBLISHED_CHUNK_MS[T]
        chunk.append({"heads": 8, "tokens": T, "ms": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
                      "tensor_tflops": round(flops / (ms / 1e3) / 1e12, 1),
                      "ascend_910b_ms": pub, "speedup_vs_ascend": round(pub / ms, 2)})
        del kw
    torch.cuda.empty_cache()
    return {"note": "the reference's published Ascend 910B shapes, raw-gate ops, per-call median after an L2 "
                    "flush; the Ascend times are other hardware, context only",
            "iters": iters, "warmup": warmup,
            "decode": decode, "verify": verify, "chunk_prefill": chunk}


# ---------------------------------------------------------------------------
# Causal-conv front end (the step before the KDA op in the attention layer)
# ---------------------------------------------------------------------------

CONV_TAPS = 4
CONV_WINDOW = 3


def conv_bytes(T: int, R: int, C: int, window: int) -> int:
    """Algorithmic bytes of one conv call: the mixed projection read and the
    q/k/v planes written (bf16), each request's window read and written, the
    fp32 weights read once."""
    return 2 * T * C * 2 + 2 * R * window * C * 2 + C * CONV_TAPS * 4


def bench_frontend(args, dist: Dist, hbm_gbs: float, steps: int, warmup: int) -> dict:
    """The causal-conv front end (``kda_causal_conv1d``: depthwise 4-tap conv
    over the mixed q|k|v projection, SiLU, q/k/v planes, conv-state window
    update) at H=32 on config 3's 8 prefill sequences (inputs larger than L2:
    no flush) and on config 2's 256 one-token decode requests (L2-sized:
    flushed per call). Per rank (weak)."""
    import kda_workloads as workloads
    import sgl_glm53_ascend_ops  # noqa: F401  (registers the torch ops)

    H = 32
    C = 3 * H * 128
    lengths = workloads.config3_lengths()
    w = workloads.conv_frontend(lengths, heads=H, window=CONV_WINDOW, seed=6000 + dist.rank, device="cuda")
    op = torch.ops.sgl_glm53_ascend.kda_causal_conv1d
    call = lambda: op(w["x"], w["weight"], None, w["conv_state"], w["cache_indices"],   # noqa: E731
                      w["query_start_loc"], None, None, None, 3, True)
    T, R = sum(lengths), len(lengths)
    ms = time_steps(call, steps, warmup, dist) / steps
    nbytes = conv_bytes(T, R, C, CONV_WINDOW)
    pre = {"workload": f"cfg3 lengths {lengths} (T={T}), C = 3 x 32 x 128 = {C}, {CONV_TAPS} taps, "
                       f"window {CONV_WINDOW}, every request continuing from its slot",
           "ms_per_step": round(ms, 4), "tokens_per_s": round(T / (ms / 1e3), 1),
           "roofline": {"bound": "hbm", "achieved": round(nbytes / (ms / 1e3) / 1e9, 1), "peak": hbm_gbs,
                        "unit": "GB/s", "frac": round(nbytes / (ms / 1e3) / 1e9 / hbm_gbs, 4),
                        "algorithmic_bytes": nbytes},
           "l2": "inputs larger than L2, no flush"}
    del w
    d = workloads.conv_frontend([1] * 256, heads=H, window=CONV_WINDOW, seed=6100 + dist.rank, device="cuda")
    dcall = lambda: op(d["x"], d["weight"], None, d["conv_state"], d["cache_indices"],   # noqa: E731
                       d["query_start_loc"], None, None, None, 3, True)
    dms = time_flushed(dcall, 20, warmup, dist)
    dbytes = conv_bytes(256, 256, C, CONV_WINDOW)
    dec = {"workload": f"cfg2 shape: 256 one-token requests, C = {C}, window {CONV_WINDOW}",
           "us": round(dms * 1e3, 2), "tokens_per_s": round(256 / (dms / 1e3), 1),
           "hbm_gbs": round(dbytes / (dms / 1e3) / 1e9, 1), "hbm_frac": round(dbytes / (dms / 1e3) / 1e9 / hbm_gbs, 4),
           "algorithmic_bytes": dbytes, "l2": "256 MiB flush before each call, median of 20"}
    del d
    torch.cuda.empty_cache()
    return {"metric": "KDA causal-conv front end (kda_causal_conv1d) tokens/s and HBM GB/s",
            "prefill": pre, "decode": dec,
            "gpu_launches_per_call": {"prefill": 2, "decode": 1},
            "launches": "prefill: conv_request_kernel + conv_stream_kernel; decode (<= 4 tokens per request on "
                        "average): conv_request_kernel alone"}


def cpu_prefill_rate(tokens: int, budget_s: float, seed: int = 8):
    """tokens/s of the CPU chunk oracle on one sequence of `tokens` tokens, H=32."""
    from oracle import kda_ref
    import kda_workloads as workloads

    threads = len(os.sched_getaffinity(0)) or 1
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
    import kda_workloads as workloads

    threads = len(os.sched_getaffinity(0)) or 1
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
    """The reference arm: the reference's own algorithm for the path on this
    host's cores. The reference is a PyTorch oracle plus Ascend-only kernels,
    so what runs here is its CPU restatement (oracle/kda_ref.py, the
    reference's kda_recur_torch with the packed-index fix), on the headline's
    exact workload: every step is all 256 requests of config 2, H=32, D=128,
    one token each, against the 512-slot pool, updated in place. Only torch,
    the oracle and the input generator are imported: no library of this
    repository is loaded into this process."""
    if dist.rank != 0:
        return
    from oracle import kda_ref
    import kda_workloads as workloads

    threads = len(os.sched_getaffinity(0)) or 1
    torch.set_num_threads(threads)
    w = workloads.config2(seed=1000)
    kw = w.kwargs()

    def step():
        kda_ref.kda_varlen_recurrent_g(**kw, out_fp32=True)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = args.steps * w.tokens / el
    sample = ("every step: all 256 requests of config 2 x 32 heads against the 512-slot pool "
              "(oracle port of the reference's kda_recur_torch, fp32)")
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "tokens/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(el / args.steps * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": DECODE_WORKLOAD, "global_batch": 256, "per_gpu_batch": 256,
                       "parallelism": "host cores (rank 0 only)"},
            "cpu_baseline": {"value": round(value, 2), "unit": "tokens/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "tokens/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------

DECODE_WORKLOAD = ("cfg2 decode: 256 req x 1 tok, H=32, K=V=128, fp32 pool 512 slots, "
                   "256 distinct slots updated in place (log-gate op)")
LINES = ("prefill", "strong", "mixed", "long", "shapes", "frontend")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--cpu-budget", type=float, default=10.0, help="seconds of CPU-oracle work")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--lines", default=",".join(LINES),
                    help="secondary lines to run besides the headline decode: " + ",".join(LINES))
    ap.add_argument("--mode", choices=("full", "kernel", "prefill-kernel", "prefill-long", "frontend-kernel"),
                    default="full",
                    help="kernel / prefill-kernel / frontend-kernel: only the timed decode / chunk / conv op "
                         "loop (profiler captures)")
    ap.add_argument("--prefill-heads", type=int, default=32,
                    help="prefill-kernel mode: heads of config 3 (fewer keeps a full ncu capture small)")
    ap.add_argument("--decode-gate", choices=("log", "raw"), default="log",
                    help="kernel mode: config 2's log-gate op, or the raw-gate op on the reference benches' inputs")
    ap.add_argument("--decode-batch", type=int, default=256, help="kernel mode: requests (1 token each), H=32")
    ap.add_argument("--prefill-path", choices=("op", "auto", "fused", "split"), default="op",
                    help="prefill-kernel mode: the torch op, or the C ABI with the chunk path forced")
    ap.add_argument("--frontend-batch", type=int, default=0,
                    help="frontend-kernel mode: 0 = config 3's prefill sequences, N = N one-token requests")
    ap.add_argument("--long-tokens", type=int, default=131072,
                    help="prefill-long mode: sequence length of config 4 (shorter keeps an ncu capture small)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    lines = {x for x in args.lines.split(",") if x}
    if not lines <= set(LINES):
        ap.error(f"--lines: unknown {sorted(lines - set(LINES))}")

    dist = Dist()
    if args.impl == "reference":
        run_reference(args, dist)
        return

    dist.init_gpu()
    bound = bind_local_cpus(dist.local)
    hbm_gbs, bf16_tf, bf16_tf_sus, peak_kind = _peaks()
    args.peaks = (hbm_gbs, bf16_tf)
    if args.mode == "prefill-kernel":
        import kda_workloads as workloads
        from sgl_glm53_ascend_ops import abi, ops
        d = workloads.config3(seed=2000 + dist.rank, heads=args.prefill_heads).to("cuda")
        kw = d.kwargs()
        if args.prefill_path == "op":
            step = lambda: ops.kda_varlen_chunk_g(**kw, prefill=True)   # noqa: E731
        else:
            path = {"auto": abi.KDA_CHUNK_AUTO, "fused": abi.KDA_CHUNK_FUSED, "split": abi.KDA_CHUNK_SPLIT}[
                args.prefill_path]
            cargs = abi.args_from_tensors(q=d.q, k=d.k, v=d.v, out=torch.empty_like(d.v), state=d.pool,
                                          indices=d.indices, cu_seqlens=d.cu_seqlens, scale=d.scale,
                                          gate_mode=abi.KDA_GATE_LOG, g=d.g, beta=d.beta)
            nws = abi.chunk_path_workspace_bytes(cargs.num_req, cargs.num_tokens, cargs.head_count, 128, path)
            ws = torch.empty(max(nws, 1), dtype=torch.uint8, device="cuda")

            def step():
                rc = abi.chunk_launch_path(cargs, ws, nws, path)
                if rc != 0:
                    raise RuntimeError(f"kda_chunk_launch_path: {abi.status_string(rc)}")
        ms = time_steps(step, args.steps, args.warmup, dist)
        if dist.rank == 0:
            print(json.dumps({"mode": "prefill-kernel", "ms_per_step": ms / args.steps}), flush=True)
        dist.close()
        return
    if args.mode == "frontend-kernel":
        import kda_workloads as workloads
        import sgl_glm53_ascend_ops  # noqa: F401
        lengths = workloads.config3_lengths() if args.frontend_batch == 0 else [1] * args.frontend_batch
        w = workloads.conv_frontend(lengths, heads=args.prefill_heads, window=CONV_WINDOW,
                                    seed=6000 + dist.rank, device="cuda")
        op = torch.ops.sgl_glm53_ascend.kda_causal_conv1d
        step = lambda: op(w["x"], w["weight"], None, w["conv_state"], w["cache_indices"],   # noqa: E731
                          w["query_start_loc"], None, None, None, 3, True)
        ms = time_steps(step, args.steps, args.warmup, dist)
        if dist.rank == 0:
            print(json.dumps({"mode": "frontend-kernel", "ms_per_step": ms / args.steps}), flush=True)
        dist.close()
        return
    if args.mode == "prefill-long":
        r = bench_prefill_long(args, dist, steps=args.steps, warmup=args.warmup)
        if dist.rank == 0:
            print(json.dumps({"mode": "prefill-long", **r}), flush=True)
        dist.close()
        return
    if args.mode == "kernel":
        import kda_workloads as workloads
        from sgl_glm53_ascend_ops import ops
        if args.decode_gate == "raw":
            # the reference's own op interface: raw gate, 1 token per request,
            # the reference benches' inputs (bench_kda_varlen_recurrent.py)
            rk = _raw_case(32, [1] * args.decode_batch, 513, seed=1000 + dist.rank)
            step = lambda: ops.kda_varlen_recurrent(**rk, prefill=False)   # noqa: E731
        else:
            kw = workloads.config2(seed=1000 + dist.rank, requests=args.decode_batch).to("cuda").kwargs()
            step = lambda: ops.kda_varlen_recurrent_g(**kw, prefill=False)   # noqa: E731
        ms = time_steps(step, args.steps, args.warmup, dist)
        if dist.rank == 0:
            print(json.dumps({"mode": "kernel", "ms_per_step": ms / args.steps}), flush=True)
        dist.close()
        return
    dec = bench_decode(args, dist, hbm_gbs, peak_kind)
    torch.cuda.empty_cache()

    extra = {}
    if "prefill" in lines:
        extra["prefill"] = bench_prefill(args, dist, hbm_gbs, bf16_tf, steps=args.prefill_steps, warmup=3)
        torch.cuda.empty_cache()
    sharded_ok = 32 % dist.world == 0
    skip_note = {"skipped": f"H=32 does not split over {dist.world} GPUs"}
    if "strong" in lines:
        extra["prefill_strong"] = (bench_prefill_strong(args, dist, hbm_gbs, bf16_tf, steps=args.prefill_steps,
                                                        warmup=3) if sharded_ok else skip_note)
    if "mixed" in lines:
        extra["mixed"] = (bench_mixed(args, dist, hbm_gbs, bf16_tf, steps=args.prefill_steps, warmup=3)
                          if sharded_ok else skip_note)
    if "long" in lines:
        extra["prefill_long"] = bench_prefill_long(args, dist, steps=20, warmup=3)
        torch.cuda.empty_cache()
    if "shapes" in lines:
        extra["published_shapes"] = bench_published_shapes(args, dist, hbm_gbs, bf16_tf, iters=20, warmup=3)
    if "frontend" in lines:
        extra["frontend"] = bench_frontend(args, dist, hbm_gbs, steps=args.prefill_steps, warmup=3)

    cpu = None
    if dist.rank == 0 and dist.world == 1:
        if bound is not None:
            os.sched_setaffinity(0, bound[0])   # the CPU baseline gets every core again
        rate, threads, sample = cpu_decode_rate(32, args.cpu_budget)
        cpu = {"value": round(rate, 2), "unit": "tokens/s", "cores": threads, "kind": "port", "sample": sample}
        if "prefill" in extra:
            prate, pthreads, psample = cpu_prefill_rate(512, args.cpu_budget)
            extra["prefill"]["cpu_baseline"] = {"value": round(prate, 2), "unit": "tokens/s", "cores": pthreads,
                                                "kind": "port", "sample": psample}

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
            "config": {"workload": DECODE_WORKLOAD,
                       "global_batch": 256 * dist.world, "per_gpu_batch": 256,
                       "l2": "inputs larger than L2 (1 GiB of state traffic per step), no flush",
                       "parallelism": f"dp{dist.world} (independent request batches, no collective)"},
            "roofline": dec["roofline"],
            "cpu_baseline": cpu,
            "e2e": dec["e2e"],
            "gpu_launches": dec["gpu_launches"],
            "clocks": dec["clocks"],
            "host_cpus": ({"bound_to_gpu_local": len(bound[1]), "of": len(bound[0])} if bound is not None
                          else "unbound (NVML gave no CPU affinity)"),
            **extra,
        }
        print(json.dumps(line), flush=True)
    dist.close()


if __name__ == "__main__":
    main()
