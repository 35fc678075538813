#!/usr/bin/env python
"""Causal multi-head attention forward+backward throughput on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 5]

Default workload (N=1): the data-parallel training-step attention — global batch 512 sequences,
T=512, d_model=768, 12 heads x head_dim 64, bf16 operands with fp32 accumulation, weights
N(0,0.02), x and dY ~ N(0,1) (seeded synthetic data).  With N GPUs (torchrun, one process per
GPU) the global batch is split evenly (512/N sequences per GPU, strong scaling) and the
Wqkv/Wo gradients are summed with one NCCL all-reduce per step.

A step is MultiHeadAttention.forward + backward over the rank's batch (QKV projection, causal
attention, output projection; projection grads, softmax VJP, dQ/dK/dV, dX), plus the gradient
all-reduce when N > 1.  ``value`` is whole-job tokens/s with inputs resident in HBM; ``e2e`` is
the same step through the public API with host (pinned) inputs: x and dY copied in, dX and the
gradients copied out, inside the timed region.  Inputs (0.8 GB each) are larger than L2.

``--impl reference`` times the reference's own NumPy path (restated in oracle/mha_oracle.py) on
this host's cores, on a bounded batch slice of the same workload.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    1: dict(name="small preset: causal MHA fwd+bwd, B=8 T=128 C=64 NH=4 D=16, fp32",
            global_batch=8, T=128, C=64, NH=4, prec="fp32", cpu_slice=8),
    2: dict(name="training batch: causal MHA fwd+bwd, B=256 T=128 C=256 NH=8 D=32, fp32 inputs, tf32 "
                 "tensor-core products", global_batch=256, T=128, C=256, NH=8, prec="tf32", cpu_slice=16),
    3: dict(name="long context: causal MHA fwd+bwd, B=32 T=1024 C=512 NH=8 D=64, bf16",
            global_batch=32, T=1024, C=512, NH=8, prec="bf16", cpu_slice=1),
    4: dict(name="generation-shaped decode: one query row per (batch, head) over an L=2048 K/V prefix, "
                 "B=64 NH=8 D=64, bf16 K/V, fp32 softmax", global_batch=64, T=2048, C=512, NH=8, prec="bf16",
            decode=True, cpu_slice=64),
    5: dict(name="data-parallel training step: causal MHA fwd+bwd, global B=512 T=512 C=768 NH=12 "
                 "D=64, bf16 operands / fp32 accumulation", global_batch=512, T=512, C=768, NH=12,
            prec="bf16", cpu_slice=2),
}
FALLBACK_PEAKS = dict(hbm_gbs=6650.0, bf16_tflops=1590.0, bf16_tflops_sustained=1400.0)


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return FALLBACK_PEAKS, "fallback"


def op_flops(op, B, T, C, NH):
    """Algorithmic FLOPs of one launch of each op of the step (no credit for recomputation)."""
    M, D = B * T, C // NH
    pairs = B * NH * T * (T + 1) // 2  # causal (query, key) pairs
    return {
        "gemm_qkv": 2 * M * 3 * C * C, "gemm_out": 2 * M * C * C, "gemm_dwo": 2 * C * C * M,
        "gemm_dctx": 2 * M * C * C, "gemm_dwqkv": 2 * C * 3 * C * M, "gemm_dx": 2 * M * C * 3 * C,
        "attn_fwd": 4 * D * pairs, "attn_bwd": 8 * D * pairs,
    }.get(op)


# ------------------------------------------------------------------------------ CPU baseline
def cpu_threads():
    try:
        from threadpoolctl import threadpool_info
        n = [i.get("num_threads", 1) for i in threadpool_info() if i.get("user_api") == "blas"]
        return max(n) if n else 1
    except Exception:
        return os.cpu_count() or 1


def cpu_step(oracle, inp, Bs, T, NH):
    import numpy as np
    out, cache = oracle.mha_forward(inp["x"], inp["w_qkv"], inp["b_qkv"], inp["w_o"], inp["b_o"], Bs, T, NH,
                                    dtype=np.float32)
    oracle.mha_backward(cache, inp["dy"], inp["w_qkv"], inp["w_o"], Bs, T, NH, dtype=np.float32)


def cpu_baseline(cfg, budget_s=12.0, max_reps=30):
    """Time the reference's NumPy forward+backward (fp32, as model/gpt.py:652-689 runs it) on a
    batch slice of the workload; best of >= 3 repetitions after one warm-up."""
    from oracle import mha_oracle as oracle
    w = WORKLOADS[cfg]
    Bs, T, C, NH = w["cpu_slice"], w["T"], w["C"], w["NH"]
    inp = oracle.make_config_inputs(cfg, Bs, T, C, NH)
    cpu_step(oracle, inp, Bs, T, NH)
    times = []
    t_start = time.perf_counter()
    while len(times) < 3 or (time.perf_counter() - t_start < budget_s and len(times) < max_reps):
        t0 = time.perf_counter()
        cpu_step(oracle, inp, Bs, T, NH)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return dict(value=Bs * T / best, unit="tokens/s", cores=cpu_threads(), kind="port",
                sample=f"{Bs} of {w['global_batch']} sequences (T={T}), fp32 NumPy forward+backward "
                       f"(oracle/mha_oracle.py restating model/gpt.py:652-689), best of {len(times)}",
                seconds_per_sample=best)


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    if WORKLOADS[cfg].get("decode"):
        w = WORKLOADS[cfg]
        base = cpu_decode_baseline(w, reps=max(args.steps, 1))
        line = dict(metric="causal attention decode tokens/sec", value=base["value"], unit="tokens/s",
                    n_gpus=args.gpus, steps=args.steps, warmup=args.warmup,
                    ms_per_step=base["seconds_per_sample"] * 1e3, higher_is_better=True, scaling="weak",
                    vs_baseline=None, dtype="f32", data="synthetic", impl="reference",
                    config=dict(workload=w["name"], batch=w["global_batch"], prefix_len=w["T"], heads=w["NH"],
                                head_dim=w["C"] // w["NH"], parallelism="host cores"),
                    cpu_baseline=base,
                    e2e=dict(value=base["value"], unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
        print(json.dumps(line), flush=True)
        return 0
    from oracle import mha_oracle as oracle
    w = WORKLOADS[cfg]
    Bs, T, C, NH = w["cpu_slice"], w["T"], w["C"], w["NH"]
    inp = oracle.make_config_inputs(cfg, Bs, T, C, NH)
    for _ in range(args.warmup):
        cpu_step(oracle, inp, Bs, T, NH)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        cpu_step(oracle, inp, Bs, T, NH)
        times.append(time.perf_counter() - t0)
    per = statistics.median(times)
    value = Bs * T / per
    line = dict(metric="causal attention fwd+bwd tokens/sec", value=value, unit="tokens/s",
                n_gpus=args.gpus, steps=args.steps, warmup=args.warmup, ms_per_step=per * 1e3,
                higher_is_better=True, scaling="strong", vs_baseline=None, dtype="f32",
                data="synthetic", impl="reference",
                config=dict(workload=w["name"], global_batch=w["global_batch"], seq_len=T, d_model=C,
                            heads=NH, head_dim=C // NH, parallelism="host cores",
                            sample_sequences_per_step=Bs),
                cpu_baseline=dict(value=value, unit="tokens/s", cores=cpu_threads(), kind="port",
                                  sample=f"{Bs} of {w['global_batch']} sequences per step, fp32 NumPy "
                                         "forward+backward (oracle/mha_oracle.py)"),
                e2e=dict(value=value, unit="tokens/s", h2d_bytes_per_step=0, d2h_bytes_per_step=0))
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------------------------ GPU helpers
class EventProfiler:
    """Named CUDA-event ranges on the current stream; sums per name after a synchronize."""

    def __init__(self):
        self.spans = []
        self.enabled = True

    class _Range:
        def __init__(self, prof, name):
            self.prof, self.name = prof, name

        def __enter__(self):
            import torch
            if self.prof.enabled:
                self.s = torch.cuda.Event(enable_timing=True)
                self.s.record()
            return self

        def __exit__(self, *exc):
            import torch
            if self.prof.enabled:
                e = torch.cuda.Event(enable_timing=True)
                e.record()
                self.prof.spans.append((self.name, self.s, e))
            return False

    def range(self, name):
        return EventProfiler._Range(self, name)

    def totals(self):
        out = {}
        for name, s, e in self.spans:
            t, n = out.get(name, (0.0, 0))
            out[name] = (t + s.elapsed_time(e), n + 1)
        return out


class _NoRange:
    def __enter__(self):
        return self

    def __exit__(self, *exc):
        return False


class MarkProfiler:
    """CUDA timing events around the named op ranges only (all ranges when ``names`` is None).
    The events are created as external events, so a range captured into a CUDA graph becomes a
    pair of event-record nodes that record again on every replay; ``last()`` then reads the
    duration of each range in the graph's latest replay."""

    def __init__(self, names=None):
        self.names = None if names is None else set(names)
        self.spans = []

    class _Range:
        def __init__(self, prof, name):
            self.prof, self.name = prof, name

        def __enter__(self):
            import torch
            self.s = torch.cuda.Event(enable_timing=True, external=True)
            self.s.record()
            return self

        def __exit__(self, *exc):
            import torch
            e = torch.cuda.Event(enable_timing=True, external=True)
            e.record()
            self.prof.spans.append((self.name, self.s, e))
            return False

    def range(self, name):
        if self.names is not None and name not in self.names:
            return _NoRange()
        return MarkProfiler._Range(self, name)

    def last(self):
        """{name: (total ms, ranges)} over the recorded ranges (after a synchronize)."""
        out = {}
        for name, s, e in self.spans:
            t, n = out.get(name, (0.0, 0))
            out[name] = (t + s.elapsed_time(e), n + 1)
        return out


class ClockSampler:
    """SM clock and clock-event (throttle) reasons sampled while the timed region runs: NVML read
    every 10 ms from a thread (read-only queries), or nvidia-smi every 200 ms where NVML is not
    importable.  The device is matched to the CUDA device by PCI bus id."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    # NVML clock-event reason bits (nvml.h: nvmlClocksEventReason*)
    BITS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []
        self.samples = []
        self.reason_bits = 0
        self.max_mhz = None
        self._nvml = None
        self._stop = threading.Event()

    def _nvml_handle(self):
        import pynvml
        pynvml.nvmlInit()
        handle = None
        try:
            import torch
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            handle = None
        if handle is None:
            handle = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        return pynvml, handle

    def start(self):
        try:
            nv, h = self._nvml_handle()
            self._nvml = (nv, h)
            self.max_mhz = float(nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM))

            def poll():
                while not self._stop.is_set():
                    try:
                        self.samples.append(float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)))
                        self.reason_bits |= int(nv.nvmlDeviceGetCurrentClocksThrottleReasons(h))
                    except Exception:
                        pass
                    self._stop.wait(0.01)
            self._t = threading.Thread(target=poll, daemon=True)
            self._t.start()
            return
        except Exception:
            self._nvml = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def stop(self):
        if self._nvml is not None:
            self._stop.set()
            self._t.join(timeout=2)
            if not self.samples:
                return None
            reasons = sorted(k for k, bit in self.BITS.items() if self.reason_bits & bit)
            return dict(sm_mhz=statistics.median(self.samples), sm_max_mhz=self.max_mhz, reasons=reasons,
                        samples=len(self.samples), source="nvml 10 ms")
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self._t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 7:
                continue
            try:
                sm.append(float(parts[0]))
                mx = float(parts[1])
            except ValueError:
                continue
            for nm, val in zip(names, parts[3:7]):
                if val.lower() in ("active", "1", "yes"):
                    reasons.add(nm)
        if not sm:
            return None
        return dict(sm_mhz=statistics.median(sm), sm_max_mhz=mx, reasons=sorted(reasons), samples=len(sm),
                    source="nvidia-smi 200 ms")


# ------------------------------------------------------------------------------ GPU arm
def run_ours(args, cfg):
    import numpy as np
    import torch
    import importlib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    pkg = importlib.import_module("llm-gpu-5_b200")
    w = dict(WORKLOADS[cfg])
    if args.batch:
        w["global_batch"] = args.batch
        w["name"] += f" [batch overridden to {args.batch}]"
    GB, T, C, NH = w["global_batch"], w["T"], w["C"], w["NH"]
    _, B = pkg.dp.shard(GB, world, rank)  # this rank's sequences (an even split of the global batch)
    M = B * T
    steps, warmup = args.steps, max(args.warmup, 3)
    use_graph = not args.eager

    np.random.seed(1000 + cfg)  # replicated weights: every rank draws the same N(0, 0.02)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=w["prec"]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + cfg + 7919 * rank)
    x = torch.randn((M, C), generator=gen, device="cuda", dtype=torch.float32)
    dy = torch.randn((M, C), generator=gen, device="cuda", dtype=torch.float32)
    reducer = None
    if dist is not None:
        attn.grad_sync_group = dist.group.WORLD
        attn.grad_buckets = args.buckets
        if not args.nccl:  # the library's NVSwitch multicast all-reduce where the GPUs support it
            reducer = pkg.dp.make_grad_reducer(attn.flat_grads.numel())
            if reducer is not None:
                if args.ar_blocks is not None:
                    reducer.max_blocks = args.ar_blocks
                if args.ar_reserve is not None:
                    reducer.reserve_sms = args.ar_reserve
                reducer.overlap = not args.ar_serial
                attn.use_grad_reducer(reducer)

    def step(xi, dyi):
        out = attn.forward(xi, B, T)
        din = attn.backward(dyi, B, T, accumulate=False)
        attn.wait_grad_sync()
        out.free()
        return din

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    align_buf = torch.zeros(1, device="cuda")

    def align():
        """After barrier(): a one-float all-reduce on the current stream, so every rank's stream
        leaves it together and the start events below are recorded at the same moment.  Without it
        the host's skew between the ranks after the barrier (up to milliseconds) is timed as step
        work by whichever rank starts first, since the first gradient all-reduce makes it wait."""
        if dist is not None:
            dist.all_reduce(align_buf)

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(warmup):
        step(x, dy).free()

    # ---------------- per-op breakdown and launches of one step (untimed)
    # every op range of the step bracketed by events; with graphs, inside a captured step's replay
    # (no host gaps between the ops), otherwise in an eager step
    l0 = pkg.launch_count()
    prof = MarkProfiler()
    attn.profiler = prof
    if use_graph:
        bd_graph = pkg.graphs.CapturedStep(lambda: step(x, dy))
        attn.profiler = None
        bd_graph.replay()
        torch.cuda.synchronize()
    else:
        step(x, dy).free()
        attn.profiler = None
        torch.cuda.synchronize()
    launches_per_step = pkg.launch_count() - l0
    totals = prof.last()
    if use_graph:
        bd_graph.reset()
    dom = max((k for k in totals if op_flops(k, B, T, C, NH)), key=lambda k: totals[k][0])

    # ---------------- eager steps: device time and host enqueue time per step
    barrier()
    align()
    h0 = time.perf_counter()
    ea, eb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ea.record()
    for _ in range(steps):
        step(x, dy).free()
    host_enqueue_ms = (time.perf_counter() - h0) * 1e3 / steps
    eb.record()
    barrier()
    eager_ms = max_over_ranks(ea.elapsed_time(eb)) / steps
    host_enqueue_ms = max_over_ranks(host_enqueue_ms)

    # ---------------- the gradient all-reduce alone (per rank, CUDA events on the launching stream)
    comm_ms = comm_ms_nccl = None
    if dist is not None:
        def time_comm(fn):
            times = []
            for _ in range(7):
                barrier()
                align()
                ca, cb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                ca.record()
                fn()
                cb.record()
                cb.synchronize()
                times.append(ca.elapsed_time(cb))
            return max_over_ranks(statistics.median(times[2:]))
        scratch = attn.flat_grads.clone()
        comm_ms_nccl = time_comm(lambda: pkg.dp.allreduce_grads(scratch, dist.group.WORLD))
        comm_ms = time_comm(reducer.allreduce) if reducer is not None else comm_ms_nccl
        del scratch

    # ---------------- timed region: captured steps replayed (or eager steps with --eager)
    # The dominant op is bracketed by timing events in every step; with graphs, R captured copies
    # of the step (sharing one memory pool) are replayed in turn, so the last R steps of the timed
    # region each leave their own reading of it.
    marks = MarkProfiler({dom})
    attn.profiler = marks
    graphs = []
    if use_graph:
        pool = torch.cuda.graph_pool_handle()
        R = max(1, min(steps, 4))
        graphs = [pkg.graphs.CapturedStep(lambda: step(x, dy), pool=pool) for _ in range(R)]
        attn.profiler = None
        for g in graphs:
            g.replay()
        run_step = lambda k: graphs[k % len(graphs)].replay()  # noqa: E731
    else:
        run_step = lambda k: step(x, dy).free()  # noqa: E731
        for k in range(2):
            run_step(k)
    clocks = ClockSampler(local)
    barrier()
    if not use_graph:
        marks.spans.clear()
    clocks.start()
    align()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    h1 = time.perf_counter()
    t0.record()
    for k in range(steps):
        run_step(k)
    host_replay_ms = (time.perf_counter() - h1) * 1e3 / steps
    t1.record()
    barrier()
    clk = clocks.stop()
    attn.profiler = None
    ms = max_over_ranks(t0.elapsed_time(t1)) / steps
    dom_t, dom_n = marks.last()[dom]
    dom_ms = max_over_ranks(dom_t / dom_n)
    value = GB * T / (ms * 1e-3)

    # ---------------- end to end through the public API with host buffers
    # Every step copies its x and dY in from pinned host memory and its dX and gradients out.  The
    # copies run on their own streams with two device slots, so step k's host->device copies overlap
    # step k-1's compute and its device->host copies (what a training loop with a prefetching data
    # loader does); each step still moves all its bytes.  With graphs each slot has its own captured
    # step reading that slot's buffers.
    x_h = torch.empty((M, C), dtype=torch.float32, pin_memory=True)
    dy_h = torch.empty((M, C), dtype=torch.float32, pin_memory=True)
    x_h.copy_(x)
    dy_h.copy_(dy)
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    slots = []
    for _ in range(2):
        sl = dict(x=torch.empty_like(x), dy=torch.empty_like(dy), g=torch.empty_like(attn.flat_grads),
                  dx_h=torch.empty((M, C), dtype=torch.float32, pin_memory=True),
                  g_h=torch.empty(attn.flat_grads.numel(), dtype=torch.float32, pin_memory=True),
                  ev_in=torch.cuda.Event(), ev_done=torch.cuda.Event(), ev_out=torch.cuda.Event(), used=False)
        sl["x"].copy_(x)
        sl["dy"].copy_(dy)
        if use_graph:
            sl["graph"] = pkg.graphs.CapturedStep(lambda sl=sl: step(sl["x"], sl["dy"]), pool=graphs[0].pool())
        slots.append(sl)
    torch.cuda.synchronize()

    def e2e_step(k):
        sl = slots[k % 2]
        with torch.cuda.stream(s_in):
            if sl["used"]:
                s_in.wait_event(sl["ev_done"])  # the slot's previous step has read its inputs
            sl["x"].copy_(x_h, non_blocking=True)
            sl["dy"].copy_(dy_h, non_blocking=True)
            sl["ev_in"].record(s_in)
        if sl["used"]:
            comp.wait_event(sl["ev_out"])  # the slot's previous results have been copied out
        comp.wait_event(sl["ev_in"])
        if use_graph:
            din = sl["graph"].replay()
            dxt = din.tensor
        else:
            din = step(sl["x"], sl["dy"])
            dxt = din.tensor
        sl["g"].copy_(attn.flat_grads)
        sl["ev_done"].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(sl["ev_done"])
            sl["dx_h"].copy_(dxt, non_blocking=True)
            sl["g_h"].copy_(sl["g"], non_blocking=True)
            sl["ev_out"].record(s_out)
        if not use_graph:
            dxt.record_stream(s_out)
            din.free()
        sl["used"] = True

    e2e_steps = max(2, min(steps, 12))
    for k in range(2):
        e2e_step(k)
    barrier()
    align()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(comp)
    s_in.wait_stream(comp)
    for k in range(e2e_steps):
        e2e_step(k)
    comp.wait_stream(s_out)
    e1.record(comp)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1)) / e2e_steps
    h2d = 2 * M * C * 4
    d2h = M * C * 4 + attn.flat_grads.numel() * 4

    # ---------------- plain pinned copies of the same bytes, all ranks at once (the host-link rate)
    link = host_link_rate(x_h, slots[0]["x"], slots[0]["dx_h"], barrier, max_over_ranks)

    for g in graphs + [sl["graph"] for sl in slots if "graph" in sl]:
        g.reset()  # graphs holding NCCL calls go before the process group
    if dist is not None:
        attn.grad_sync_group = None
        dist.barrier()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return 0

    # ---------------- the line
    peaks, src = load_peaks()
    per_op = {k: dict(ms_per_step=t, ranges_per_step=n) for k, (t, n) in totals.items()}
    achieved = op_flops(dom, B, T, C, NH) / (dom_ms * 1e-3) / 1e12
    peak, peak_src, bound = precision_peak(w["prec"], peaks, src)
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            full = json.load(f).get(f"cfg{cfg}", {}).get(dom)
        # recorded for the whole global batch on one GPU; every sequence is independent work, so
        # a launch over this rank's B sequences moves B / global_batch of it
        if full is not None and not args.batch:
            traffic = full * B / GB
    tflops = group_tflops(totals, lambda k: op_flops(k, B, T, C, NH))
    copy_gbs = (h2d + d2h) * world / (e2e_ms * 1e-3) / 1e9
    # the step's copies alone at the measured link rates: the slowest of each direction by itself
    # and both directions together
    link_ms = 1e3 * max(h2d * world / (link["h2d_gbs"] * 1e9), d2h * world / (link["d2h_gbs"] * 1e9),
                        (h2d + d2h) * world / (link["duplex_gbs"] * 1e9))
    line = dict(
        metric="causal attention fwd+bwd tokens/sec", value=value, unit="tokens/s", n_gpus=world,
        steps=steps, warmup=warmup, ms_per_step=ms, higher_is_better=True, scaling="strong",
        vs_baseline=None, dtype=DTYPE_NAME[w["prec"]], data="synthetic",
        config=dict(workload=w["name"], global_batch=GB, seq_len=T, d_model=C, heads=NH, head_dim=C // NH,
                    per_gpu_batch=B, parallelism=f"dp{world}", l2="inputs larger than L2 (no flush)",
                    launch="CUDA graph: the step captured once, replayed" if use_graph else "eager"),
        roofline=dict(bound=bound, kernel=dom, achieved=achieved, peak=peak, unit="TFLOP/s",
                      frac=achieved / peak, traffic=traffic,
                      peak_source=f"{peak_src}; the timed region is {ms * steps / 1e3:.2f} s",
                      frac_of_sustained=(achieved / peaks.get("bf16_tflops_sustained",
                                                              FALLBACK_PEAKS["bf16_tflops_sustained"])
                                         if w["prec"] == "bf16" else None)),
        step_tflops=sum(op_flops(k, B, T, C, NH) or 0 for k in totals) * world / (ms * 1e-3) / 1e12,
        tflops=tflops,
        breakdown=per_op,
        timing=dict(eager_ms_per_step=eager_ms, host_enqueue_ms_eager=host_enqueue_ms,
                    host_enqueue_ms_graph=host_replay_ms if use_graph else None, comm_ms=comm_ms,
                    comm_ms_nccl=comm_ms_nccl, comm_bytes=attn.flat_grads.numel() * 4 if dist is not None else 0,
                    grad_sync=None if dist is None else (
                        (f"NVSwitch multicast all-reduce kernel (attn_grad_allreduce), {reducer.max_blocks} "
                         f"CTAs beside the dX GEMM on {reducer.reserve_sms} SMs it leaves free"
                         if reducer is not None else "NCCL all_reduce")
                        + ("; two buckets: dWo/dbo after the dWo GEMM, dWqkv/dbqkv after the dWqkv GEMM"
                           if attn.grad_buckets else "; one bucket after the dWqkv GEMM")),
                    note="eager: the same step launched op by op from Python; comm_ms: the step's gradient "
                         "all-reduce alone, comm_ms_nccl: NCCL's on the same buffer, medians of 5, max over "
                         "ranks; every timed region starts after a barrier and a one-float all-reduce on the "
                         "timed stream, so the ranks' start events are recorded together"),
        gpu_launches=launches_per_step * steps,
        e2e=dict(value=GB * T / (e2e_ms * 1e-3), unit="tokens/s", h2d_bytes_per_step=h2d * world,
                 d2h_bytes_per_step=d2h * world, ms_per_step=e2e_ms, copy_gbs=copy_gbs,
                 host_link_gbs=link, link_bound_ms=link_ms, frac_of_link_bound=link_ms / e2e_ms),
        clocks=clk,
    )
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    if world == 1 and not args.no_configs and not args.batch:
        line["configs"] = measure_other_configs(args, pkg, peaks, src)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def group_tflops(totals, flops_of):
    """Attention core (QK^T, PV, dP, dV, dQ, dK: 12*D per causal pair, no credit for recomputing
    S) and projection GEMMs, each over its own event-timed ranges, and their sum.  ``totals`` maps an
    op to (ms in one step, ranges in one step); ``flops_of`` gives one range's FLOPs."""
    groups = {}
    for k, (t, n) in totals.items():
        f = flops_of(k)
        if f:
            g = "attention_core" if k.startswith("attn_") else "projections"
            fl, tm = groups.get(g, (0, 0.0))
            groups[g] = (fl + f * n, tm + t)
    out = {g: dict(tflop_per_step=fl / 1e12, ms_per_step=tm, tflops=fl / (tm * 1e-3) / 1e12)
           for g, (fl, tm) in groups.items()}
    if groups:
        fl = sum(v[0] for v in groups.values())
        tm = sum(v[1] for v in groups.values())
        out["sum"] = dict(tflop_per_step=fl / 1e12, ms_per_step=tm, tflops=fl / (tm * 1e-3) / 1e12)
    return out


def host_link_rate(h_src, d_buf, h_dst, barrier, max_over_ranks, reps=3):
    """Plain pinned copies of one step-sized buffer, every rank at once: host->device, device->host,
    and both together on two streams.  GB/s summed over the ranks (all ranks' bytes / the slowest
    rank's time), best of ``reps``."""
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    nb = h_src.numel() * h_src.element_size()
    cur = torch.cuda.current_stream()
    other = torch.cuda.Stream()
    d2 = torch.empty_like(d_buf)
    res = {}
    for name in ("h2d", "d2h", "duplex"):
        best = None
        for _ in range(reps):
            barrier()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(cur)
            if name == "duplex":  # the device->host copy starts with the host->device one
                other.wait_event(a)
                with torch.cuda.stream(other):
                    h_dst.copy_(d2, non_blocking=True)
            if name in ("h2d", "duplex"):
                d_buf.copy_(h_src, non_blocking=True)
            if name == "d2h":
                h_dst.copy_(d2, non_blocking=True)
            if name == "duplex":
                cur.wait_stream(other)
            b.record(cur)
            b.synchronize()
            t = max_over_ranks(a.elapsed_time(b))
            best = t if best is None else min(best, t)
        moved = nb * (2 if name == "duplex" else 1) * world
        res[f"{name}_gbs"] = moved / (best * 1e-3) / 1e9
    res["bytes_per_rank"] = nb
    return res


# ------------------------------------------------------------------------------ the other configs
def fp32_core_peak(peaks):
    """FP32 CUDA-core peak of the GPU, derived (no measured FP32 figure exists): SMs x 128 FP32 lanes
    x 2 FLOP per FMA x the measured maximum SM clock."""
    import torch
    sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    mhz = peaks.get("sm_max_mhz", 1965.0)
    return sms * 128 * 2 * mhz * 1e6 / 1e12, f"derived: {sms} SMs x 128 lanes x 2 x {mhz:.0f} MHz"


DTYPE_NAME = dict(bf16="bf16", tf32="tf32", fp32="f32")


def precision_peak(prec, peaks, src):
    """(peak TFLOP/s, where it comes from, bound) for a step computed in ``prec``: bf16 the measured
    burst bf16 figure; tf32 half of it (the dense tf32 rate is half the bf16 rate on this part; no
    tf32 figure is measured); fp32 the CUDA-core peak."""
    if prec == "bf16":
        return peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]), f"{src} bf16_tflops (burst)", "tensor"
    if prec == "tf32":
        return (peaks.get("bf16_tflops", FALLBACK_PEAKS["bf16_tflops"]) / 2,
                f"derived: half of the {src} bf16_tflops (burst)", "tensor")
    peak, psrc = fp32_core_peak(peaks)
    return peak, psrc, "fp32 CUDA core"


def measure_module_config(args, pkg, cfg, peaks, src, prec=None):
    """MultiHeadAttention forward + backward at one configuration's full size on one GPU: the step
    captured as a CUDA graph, each replay timed with events after a 256 MB write that flushes L2,
    every op range timed inside the replays.  ``prec`` overrides the configuration's precision."""
    import numpy as np
    import torch
    w = dict(WORKLOADS[cfg])
    if prec is not None and prec != w["prec"]:
        w["prec"] = prec
        w["name"] = w["name"].split(", fp32 inputs")[0] + f", {prec}"
    B, T, C, NH = w["global_batch"], w["T"], w["C"], w["NH"]
    steps = max(args.steps, 3)
    np.random.seed(1000 + cfg)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=w["prec"]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + cfg)
    x = torch.randn((B * T, C), generator=gen, device="cuda")
    dy = torch.randn((B * T, C), generator=gen, device="cuda")

    def step():
        out = attn.forward(x, B, T)
        din = attn.backward(dy, B, T)
        attn.wait_grad_sync()
        out.free()
        return din

    for _ in range(max(args.warmup, 3)):
        step().free()
    prof = MarkProfiler()
    attn.profiler = prof
    graph = pkg.graphs.CapturedStep(step)
    attn.profiler = None
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")  # 256 MB, twice the L2
    times, optot = [], {}
    for k in range(steps + 1):
        flush.zero_()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        if k == 0:
            continue  # the first replay uploads the graph
        times.append(a.elapsed_time(b))
        for name, (t, n) in prof.last().items():
            s = optot.setdefault(name, [0.0, n])
            s[0] += t
    graph.reset()
    ms = statistics.median(times)
    totals = {name: (t / steps, n) for name, (t, n) in optot.items()}
    flops_of = lambda k: op_flops(k, B, T, C, NH)  # noqa: E731
    dom = max((k for k in totals if flops_of(k)), key=lambda k: totals[k][0])
    dom_ach = flops_of(dom) / (totals[dom][0] / totals[dom][1] * 1e-3) / 1e12
    peak, psrc, bound = precision_peak(w["prec"], peaks, src)
    tflops = group_tflops(totals, flops_of)
    for g in tflops.values():
        g["frac"] = g["tflops"] / peak
    res = dict(workload=w["name"], value=B * T / (ms * 1e-3), unit="tokens/s", ms_per_step=ms,
               dtype=DTYPE_NAME[w["prec"]], steps=steps, tflops=tflops,
               roofline=dict(bound=bound, kernel=dom,
                             achieved=dom_ach, peak=peak, unit="TFLOP/s", frac=dom_ach / peak, peak_source=psrc),
               breakdown={k: dict(ms_per_step=t, ranges_per_step=n) for k, (t, n) in totals.items()},
               l2="a 256 MB buffer written before every timed step (L2 flushed)",
               launch="CUDA graph: the step captured once, replayed")
    del attn, x, dy, flush
    torch.cuda.empty_cache()
    if not args.no_cpu_baseline:
        res["cpu_baseline"] = cpu_baseline(cfg, budget_s=6.0)
    return res


def measure_other_configs(args, pkg, peaks, src):
    """Configurations 1-4 at full size on one GPU, each with its CPU baseline; a configuration that
    fails reports its error instead of a number."""
    out = {}
    # configuration 2 in both float32 arithmetics: tf32 products (its line) and exact fp32
    for key, cfg, prec in (("cfg1", 1, None), ("cfg2", 2, None), ("cfg2_fp32", 2, "fp32"), ("cfg3", 3, None),
                           ("cfg4", 4, None)):
        try:
            if WORKLOADS[cfg].get("decode"):
                out[key] = decode_line(args, cfg, pkg, world=1, rank=0)
            else:
                out[key] = measure_module_config(args, pkg, cfg, peaks, src, prec)
        except Exception as e:  # reported in the line; the headline number stands on its own
            out[key] = dict(workload=WORKLOADS[cfg]["name"], error=f"{type(e).__name__}: {e}"[:300])
    return out


# ------------------------------------------------------------------------------ decode (cfg 4)
def decode_inputs(B, NH, L, D, seed):
    import numpy as np
    rng = np.random.default_rng(seed)
    return [rng.standard_normal(shape).astype(np.float32) for shape in ((B, NH, D), (B, L, NH, D), (B, L, NH, D))]


def cpu_decode_baseline(w, reps=5):
    """The oracle's float32 NumPy decode (oracle.decode_attention) over the whole workload."""
    import numpy as np
    from oracle import mha_oracle as oracle
    B, L, NH = w["global_batch"], w["T"], w["NH"]
    D = w["C"] // NH
    q, k, v = decode_inputs(B, NH, L, D, 1004)
    kt, vt = k.transpose(0, 2, 1, 3), v.transpose(0, 2, 1, 3)
    oracle.decode_attention(q, kt, vt, 1.0 / D ** 0.5, dtype=np.float32)
    times = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.decode_attention(q, kt, vt, 1.0 / D ** 0.5, dtype=np.float32)
        times.append(time.perf_counter() - t0)
    best = min(times)
    return dict(value=B / best, unit="tokens/s", cores=cpu_threads(), kind="port",
                sample=f"the whole step ({B} sequences x {NH} heads over L={L}), fp32 NumPy "
                       f"(oracle/mha_oracle.py decode_attention), best of {reps}",
                seconds_per_sample=best)


def run_decode(args, cfg):
    import torch
    import importlib
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
    pkg = importlib.import_module("llm-gpu-5_b200")
    line = decode_line(args, cfg, pkg, world, rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def decode_line(args, cfg, pkg, world, rank):
    """One decode step = one attn_decode call for B sequences; inputs (q and two alternating
    copies of the K/V cache, 268 MB each, so no call reads L2-resident data) are on the device.
    Returns the JSON line (replicas: each GPU runs its own batch, no collective)."""
    import torch
    local = torch.cuda.current_device()
    w = WORKLOADS[cfg]
    B, L, NH = args.batch or w["global_batch"], w["T"], w["NH"]
    D = w["C"] // NH
    steps, warmup = args.steps, max(args.warmup, 3)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1004 + 7919 * rank)
    q = torch.randn((B, NH, D), generator=gen, device="cuda").to(torch.bfloat16)
    caches = [(torch.randn((B, L, NH, D), generator=gen, device="cuda").to(torch.bfloat16),
               torch.randn((B, L, NH, D), generator=gen, device="cuda").to(torch.bfloat16)) for _ in range(2)]
    out = torch.empty_like(q)
    lse = torch.empty((B, NH), dtype=torch.float32, device="cuda")
    ws = torch.empty(pkg.lib.attn_decode_workspace_size(B, NH, L, D), dtype=torch.uint8, device="cuda")

    def step(i):
        k, v = caches[i & 1]
        pkg.mha_ops.decode(q, k, v, out=out, lse=lse, workspace=ws)

    for i in range(warmup):
        step(i)
    clocks = ClockSampler(local)
    torch.cuda.synchronize()
    clocks.start()
    launches0 = pkg.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for i in range(steps):
        step(i)
    t1.record()
    torch.cuda.synchronize()
    launches = pkg.launch_count() - launches0
    clk = clocks.stop()
    ms = t0.elapsed_time(t1) / steps
    # end to end through the public API: q from pinned host memory, the output back to the host
    q_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    o_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    q_h.copy_(q)
    for i in range(2):
        q.copy_(q_h, non_blocking=True)
        step(i)
        o_h.copy_(out, non_blocking=True)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(steps):
        q.copy_(q_h, non_blocking=True)
        step(i)
        o_h.copy_(out, non_blocking=True)
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = e0.elapsed_time(e1) / steps
    if rank != 0:
        return None
    peaks, src = load_peaks()
    kv_bytes = 2 * B * L * NH * D * 2
    achieved = kv_bytes / (ms * 1e-3) / 1e9
    peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
    line = dict(
        metric="causal attention decode tokens/sec", value=B * world / (ms * 1e-3), unit="tokens/s",
        n_gpus=world, steps=steps, warmup=warmup, ms_per_step=ms, higher_is_better=True, scaling="weak",
        vs_baseline=None, dtype="bf16", data="synthetic",
        config=dict(workload=w["name"], batch=B, prefix_len=L, heads=NH, head_dim=D,
                    parallelism="replicas" if world > 1 else "single GPU",
                    l2="two alternating 268 MB K/V caches (larger than L2)"),
        roofline=dict(bound="hbm", kernel="attn_decode", achieved=achieved, peak=peak, unit="GB/s",
                      frac=achieved / peak, traffic=None, peak_source=f"{src} hbm_gbs",
                      algorithmic_bytes=kv_bytes),
        gpu_launches=launches,
        e2e=dict(value=B * world / (e2e_ms * 1e-3), unit="tokens/s", h2d_bytes_per_step=q.numel() * 2 * world,
                 d2h_bytes_per_step=out.numel() * 2 * world, ms_per_step=e2e_ms),
        clocks=clk,
    )
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_baseline(w)
    return line


# ------------------------------------------------------------------------------ fused half-block
def run_residual(args, cfg):
    """x += attn(ln_1(x)), the pre-attention half of TransformerBlock (model/gpt.py:778-783 forward,
    :823-838 backward), timed two ways on the same inputs: the reference's sequence with this
    library's kernels (LayerNorm to float32, MultiHeadAttention.forward, residual add; backward:
    attn.backward, the LayerNorm backward to its own buffer, the residual add) and the fused
    forward_residual / backward_residual.  Forward alone (inference) and forward + backward."""
    import numpy as np
    import torch
    import importlib
    pkg = importlib.import_module("llm-gpu-5_b200")
    ops = pkg.mha_ops
    w = WORKLOADS[cfg]
    B = args.batch or w["global_batch"]
    T, C, NH = w["T"], w["C"], w["NH"]
    M = B * T
    np.random.seed(1000 + cfg)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=w["prec"]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + cfg)
    x0 = torch.randn((M, C), generator=gen, device="cuda")
    dy0 = torch.randn((M, C), generator=gen, device="cuda")
    gamma = 1 + 0.1 * torch.randn(C, generator=gen, device="cuda")
    beta = 0.1 * torch.randn(C, generator=gen, device="cuda")
    dgamma, dbeta = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    x, dy = x0.clone(), dy0.clone()

    def unfused_fwd():
        ln = ops.layernorm(x, gamma, beta)
        out = attn.forward(ln, B, T)
        x.add_(out.tensor)
        out.free()

    def fused_fwd():
        attn.forward_residual(x, B, T, gamma, beta)

    def unfused_step():
        x_in = x.clone()  # cache_input_ln1 (model/gpt.py:773-775)
        unfused_fwd()
        dln = attn.backward(dy, B, T)
        dxn = torch.empty_like(x)
        ops.layernorm_backward(dln.tensor.view(M, C), x_in, gamma, dxn, dgamma, dbeta)
        dx0 = dy.clone()  # dX0 = dX1 + dLN (model/gpt.py:833-835)
        dx0.add_(dxn)
        dln.free()

    def fused_step():
        attn.forward_residual(x, B, T, gamma, beta)
        attn.backward_residual(dy, B, T, gamma, dgamma, dbeta)

    res = {}
    for name, fn, training in (("unfused_fwd", unfused_fwd, False), ("fused_fwd", fused_fwd, False),
                               ("unfused_fwd_bwd", unfused_step, True), ("fused_fwd_bwd", fused_step, True)):
        attn.training = training
        for _ in range(max(args.warmup, 3)):
            x.copy_(x0)
            dy.copy_(dy0)
            fn()
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        total = 0.0
        for _ in range(args.steps):  # x and dY are reset outside the timed spans
            x.copy_(x0)
            dy.copy_(dy0)
            t0.record()
            fn()
            t1.record()
            torch.cuda.synchronize()
            total += t0.elapsed_time(t1)
        res[name] = total / args.steps
    print(json.dumps(dict(metric="pre-attention half-block fwd+bwd tokens/sec",
                          value=M / (res["fused_fwd_bwd"] * 1e-3), unit="tokens/s",
                          ms=res, speedup_fwd=res["unfused_fwd"] / res["fused_fwd"],
                          speedup_fwd_bwd=res["unfused_fwd_bwd"] / res["fused_fwd_bwd"],
                          dtype="bf16" if w["prec"] == "bf16" else "f32",
                          data="synthetic", config=dict(workload=w["name"], tokens=M))), flush=True)
    return 0


# ------------------------------------------------------------------------------ feed-forward block
def ffn_op_flops(op, M, C):
    H = 4 * C
    return 2 * M * C * H if op in ("gemm_fc_gelu", "gemm_proj", "gemm_dwproj", "gemm_dhidden_gelu", "gemm_dwfc",
                                   "gemm_dx") else None


def run_ffn(args, cfg):
    """FeedForward forward + backward (model/gpt.py:327-456) at the workload's token count and
    d_model (hidden 4 x d_model), bf16 operands / fp32 accumulation: six tcgen05 GEMMs, GELU and its
    derivative in their epilogues.  Prints one JSON line with per-op times and TFLOP/s against the
    measured bf16 peak, and, for context, the same computation as cuBLAS GEMMs plus PyTorch's
    tanh-GELU kernels (torch.matmul, F.gelu, aten.gelu_backward, column sums)."""
    import numpy as np
    import torch
    import torch.nn.functional as F
    import importlib
    pkg = importlib.import_module("llm-gpu-5_b200")
    w = WORKLOADS[cfg]
    B = args.batch or w["global_batch"]
    T, C = w["T"], w["C"]
    M, H = B * T, 4 * w["C"]
    steps, warmup = args.steps, max(args.warmup, 3)
    np.random.seed(1000 + cfg)
    ffn = pkg.FeedForward(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=w["NH"], max_len=T,
                                        attention_precision=w["prec"]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(2000 + cfg)
    for p in (ffn.c_fc_b, ffn.c_proj_b):
        p.weights.copy_(0.1 * torch.randn(p.shape, generator=gen, device="cuda"))
    x = torch.randn((M, C), generator=gen, device="cuda")
    dy = torch.randn((M, C), generator=gen, device="cuda")

    def step():
        out = ffn.forward(x, B, T)
        din = ffn.backward(dy, B, T)
        out.free()
        din.free()

    for _ in range(warmup):
        step()
    prof = EventProfiler()
    ffn.profiler = prof
    step()
    prof.spans.clear()
    clocks = ClockSampler(0)
    torch.cuda.synchronize()
    clocks.start()
    launches0 = pkg.launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    clk = clocks.stop()
    launches = pkg.launch_count() - launches0
    ms = t0.elapsed_time(t1) / steps
    ffn.profiler = None
    totals = prof.totals()
    peaks, src = load_peaks()
    peak = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    per_op = {}
    for k, (t, n) in totals.items():
        d = dict(ms_per_step=t / steps, launches_per_step=n / steps)
        f = ffn_op_flops(k, M, C)
        if f:
            d["tflops"] = f / (t / n * 1e-3) / 1e12
        per_op[k] = d
    gemm_flops = 12 * M * C * H
    gemm_ms = sum(totals[k][0] for k in totals if ffn_op_flops(k, M, C)) / steps
    dom = max((k for k in totals if ffn_op_flops(k, M, C)), key=lambda k: totals[k][0])
    dom_ach = ffn_op_flops(dom, M, C) / (totals[dom][0] / totals[dom][1] * 1e-3) / 1e12

    # the same math on NVIDIA's libraries (bf16 everywhere; context only)
    xb, dyb = x.bfloat16(), dy.bfloat16()
    wfc, wpr = ffn.c_fc_w.weights.bfloat16(), ffn.c_proj_w.weights.bfloat16()
    bfc, bpr = ffn.c_fc_b.weights.bfloat16(), ffn.c_proj_b.weights.bfloat16()

    def vendor_step():
        pre = torch.addmm(bfc, xb, wfc)
        act = F.gelu(pre, approximate="tanh")
        torch.addmm(bpr, act, wpr)
        act.t() @ dyb
        dyb.sum(0)
        dpre = torch.ops.aten.gelu_backward(dyb @ wpr.t(), pre, approximate="tanh")
        xb.t() @ dpre
        dpre.sum(0)
        dpre @ wfc.t()

    for _ in range(warmup):
        vendor_step()
    torch.cuda.synchronize()
    v0, v1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    v0.record()
    for _ in range(steps):
        vendor_step()
    v1.record()
    torch.cuda.synchronize()
    vendor_ms = v0.elapsed_time(v1) / steps
    print(json.dumps(dict(
        metric="feed-forward fwd+bwd tokens/sec", value=M / (ms * 1e-3), unit="tokens/s", n_gpus=1, steps=steps,
        warmup=warmup, ms_per_step=ms, higher_is_better=True, dtype="bf16" if w["prec"] == "bf16" else "f32",
        data="synthetic",
        config=dict(workload=f"FeedForward fwd+bwd, {M} tokens (B={B} T={T}), C={C} -> {H} -> {C}, tanh-GELU",
                    tokens=M, d_model=C, hidden=H, l2="inputs larger than L2 (no flush)"),
        roofline=dict(bound="tensor", kernel=dom, achieved=dom_ach, peak=peak, unit="TFLOP/s", frac=dom_ach / peak,
                      peak_source=f"{src} bf16_tflops_sustained"),
        gemm_tflops=gemm_flops / (gemm_ms * 1e-3) / 1e12, step_tflops=gemm_flops / (ms * 1e-3) / 1e12,
        breakdown=per_op, gpu_launches=launches, clocks=clk,
        vendor=dict(cublas_plus_torch_gelu_ms=vendor_ms, speedup=vendor_ms / ms))), flush=True)
    return 0


# ------------------------------------------------------------------------------ vendor libraries
def run_vendor(args, cfg):
    """Time NVIDIA's own B200 kernels on the same workload, for context: cuDNN attention through
    torch.nn.functional.scaled_dot_product_attention (causal, bf16, [B, NH, T, D]) and cuBLAS
    through torch.matmul for the six projection GEMMs.  Prints one JSON line; not a bench line."""
    import torch
    import torch.nn.functional as F
    from torch.nn.attention import sdpa_kernel, SDPBackend
    w = WORKLOADS[cfg]
    B = args.batch or w["global_batch"]
    T, C, NH = w["T"], w["C"], w["NH"]
    D, M = C // NH, B * T
    torch.manual_seed(0)

    def timed(fn, reps=max(args.steps, 3)):
        for _ in range(max(args.warmup, 3)):
            fn()
        torch.cuda.synchronize()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record()
        for _ in range(reps):
            fn()
        s1.record()
        torch.cuda.synchronize()
        return s0.elapsed_time(s1) / reps

    out = dict(workload=w["name"], batch=B)
    q, k, v = (torch.randn(B, NH, T, D, device="cuda", dtype=torch.bfloat16).requires_grad_() for _ in range(3))
    do = torch.randn(B, NH, T, D, device="cuda", dtype=torch.bfloat16)
    for name, be in (("cudnn", SDPBackend.CUDNN_ATTENTION), ("flash", SDPBackend.FLASH_ATTENTION)):
        try:
            with sdpa_kernel(be):
                fwd = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True))
                both = timed(lambda: F.scaled_dot_product_attention(q, k, v, is_causal=True).backward(do))
            out[f"sdpa_{name}_fwd_ms"] = fwd
            out[f"sdpa_{name}_fwd_bwd_ms"] = both
        except Exception as e:  # a backend that does not support the shape on this build
            out[f"sdpa_{name}"] = f"unavailable: {str(e).splitlines()[0][:120]}"
    del q, k, v, do
    x = torch.randn(M, C, device="cuda", dtype=torch.bfloat16)
    wq = torch.randn(C, 3 * C, device="cuda", dtype=torch.bfloat16)
    wo = torch.randn(C, C, device="cuda", dtype=torch.bfloat16)
    g3 = torch.randn(M, 3 * C, device="cuda", dtype=torch.bfloat16)
    g1 = torch.randn(M, C, device="cuda", dtype=torch.bfloat16)
    gemms = dict(gemm_qkv=lambda: x @ wq, gemm_out=lambda: g1 @ wo, gemm_dwo=lambda: g1.t() @ g1,
                 gemm_dctx=lambda: g1 @ wo.t(), gemm_dwqkv=lambda: x.t() @ g3, gemm_dx=lambda: g3 @ wq.t())
    for name, fn in gemms.items():
        out[f"cublas_{name}_ms"] = timed(fn)
    print(json.dumps(dict(vendor=out)), flush=True)
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference", "vendor"], default="ours",
                    help="vendor: time cuDNN attention and cuBLAS GEMMs on the same workload (context only)")
    ap.add_argument("--config", type=int, default=5, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", action="store_true",
                    help="leave out the 'configs' object (configurations 1-4 measured after the headline)")
    ap.add_argument("--nccl", action="store_true",
                    help="sum the gradients with NCCL instead of the library's NVSwitch multicast all-reduce")
    ap.add_argument("--buckets", action="store_true",
                    help="all-reduce dWo/dbo right after the dWo GEMM and dWqkv/dbqkv after the dWqkv GEMM "
                         "(default: one bucket after the dWqkv GEMM)")
    ap.add_argument("--ar-blocks", type=int, default=None,
                    help="CTAs of the multicast all-reduce (default: the reducer's, 16)")
    ap.add_argument("--ar-reserve", type=int, default=None,
                    help="SMs the dX GEMM leaves to the multicast all-reduce beside it (default: the "
                         "reducer's, 16; 0: none)")
    ap.add_argument("--ar-serial", action="store_true",
                    help="run the multicast all-reduce after the input-gradient GEMM instead of beside it")
    ap.add_argument("--eager", action="store_true",
                    help="launch every step op by op from Python instead of replaying a captured CUDA graph")
    ap.add_argument("--residual", action="store_true",
                    help="time x += attn(ln_1(x)) fused (forward_residual) against the unfused block sequence")
    ap.add_argument("--ffn", action="store_true",
                    help="time FeedForward fwd+bwd (C -> 4C -> C) at the workload's token count and d_model")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the global batch (small cases for profiler captures only)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args, args.config)
    if args.impl == "vendor":
        return run_vendor(args, args.config)
    if WORKLOADS[args.config].get("decode"):
        return run_decode(args, args.config)
    if args.residual:
        return run_residual(args, args.config)
    if args.ffn:
        return run_ffn(args, args.config)
    return run_ours(args, args.config)


if __name__ == "__main__":
    sys.exit(main())
