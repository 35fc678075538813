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
    2: dict(name="training batch: causal MHA fwd+bwd, B=256 T=128 C=256 NH=8 D=32, fp32",
            global_batch=256, T=128, C=256, NH=8, prec="fp32", cpu_slice=16),
    3: dict(name="long context: causal MHA fwd+bwd, B=32 T=1024 C=512 NH=8 D=64, bf16",
            global_batch=32, T=1024, C=512, NH=8, prec="bf16", cpu_slice=1),
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


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def start(self):
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
        return dict(sm_mhz=statistics.median(sm), sm_max_mhz=mx, reasons=sorted(reasons), samples=len(sm))


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

    np.random.seed(1000 + cfg)  # replicated weights: every rank draws the same N(0, 0.02)
    attn = pkg.MultiHeadAttention(pkg.GPTConfig(vocab_size=50, embedding_dim=C, num_heads=NH, max_len=T,
                                                attention_precision=w["prec"]))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1000 + cfg + 7919 * rank)
    x = torch.randn((M, C), generator=gen, device="cuda", dtype=torch.float32)
    dy = torch.randn((M, C), generator=gen, device="cuda", dtype=torch.float32)
    if dist is not None:
        attn.grad_sync_group = dist.group.WORLD

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

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-resident timing
    for _ in range(warmup):
        step(x, dy).free()
    prof = EventProfiler()
    attn.profiler = prof
    step(x, dy).free()  # one profiled step outside the timed region primes the event objects
    prof.spans.clear()
    clocks = ClockSampler(local)
    barrier()
    clocks.start()
    launches0 = pkg.launch_count()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step(x, dy).free()
    t1.record()
    barrier()
    clk = clocks.stop()
    launches = pkg.launch_count() - launches0
    ms = max_over_ranks(t0.elapsed_time(t1)) / steps
    attn.profiler = None
    totals = prof.totals()
    value = GB * T / (ms * 1e-3)

    # ---------------- end to end through the public API with host buffers
    # Every step copies its x and dY in from pinned host memory and its dX and gradients out.
    # The copies run on their own streams with double-buffered device slots, so step k's
    # host->device copies overlap step k-1's compute and step k-1's device->host copies (what a
    # training loop with a prefetching data loader does); each step still moves all its bytes.
    x_h = torch.empty((M, C), dtype=torch.float32, pin_memory=True)
    dy_h = torch.empty((M, C), dtype=torch.float32, pin_memory=True)
    x_h.copy_(x)
    dy_h.copy_(dy)
    comp = torch.cuda.current_stream()
    s_in, s_out = torch.cuda.Stream(), torch.cuda.Stream()
    slots = []
    for _ in range(2):
        slots.append(dict(
            x=torch.empty_like(x), dy=torch.empty_like(dy),
            g=torch.empty_like(attn.flat_grads),
            dx_h=torch.empty((M, C), dtype=torch.float32, pin_memory=True),
            g_h=torch.empty(attn.flat_grads.numel(), dtype=torch.float32, pin_memory=True),
            ev_x=torch.cuda.Event(), ev_dy=torch.cuda.Event(), ev_done=torch.cuda.Event(),
            ev_out=torch.cuda.Event(), used=False))

    def e2e_step(k):
        sl = slots[k % 2]
        with torch.cuda.stream(s_in):
            if sl["used"]:
                s_in.wait_event(sl["ev_done"])  # the slot's previous step has read its inputs
            sl["x"].copy_(x_h, non_blocking=True)
            sl["ev_x"].record(s_in)
            sl["dy"].copy_(dy_h, non_blocking=True)
            sl["ev_dy"].record(s_in)
        if sl["used"]:
            comp.wait_event(sl["ev_out"])  # the slot's previous gradient snapshot has been copied out
        comp.wait_event(sl["ev_x"])
        out = attn.forward(sl["x"], B, T)
        comp.wait_event(sl["ev_dy"])
        din = attn.backward(sl["dy"], B, T)
        attn.wait_grad_sync()
        sl["g"].copy_(attn.flat_grads)
        sl["ev_done"].record(comp)
        with torch.cuda.stream(s_out):
            s_out.wait_event(sl["ev_done"])
            sl["dx_h"].copy_(din.tensor, non_blocking=True)
            sl["g_h"].copy_(sl["g"], non_blocking=True)
            sl["ev_out"].record(s_out)
        din.tensor.record_stream(s_out)
        sl["used"] = True
        out.free()
        din.free()

    e2e_steps = max(2, min(steps, 6))
    for k in range(2):
        e2e_step(k)
    barrier()
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

    if dist is not None:
        attn.grad_sync_group = None
        dist.barrier()
    if rank != 0:
        if dist is not None:
            dist.destroy_process_group()
        return 0

    # ---------------- roofline of the dominant kernel
    peaks, src = load_peaks()
    per_op = {k: dict(ms_per_step=t / steps, launches_per_step=n / steps) for k, (t, n) in totals.items()}
    dom = max((k for k in totals if op_flops(k, B, T, C, NH)), key=lambda k: totals[k][0])
    dom_ms = totals[dom][0] / totals[dom][1]
    achieved = op_flops(dom, B, T, C, NH) / (dom_ms * 1e-3) / 1e12
    peak = peaks.get("bf16_tflops_sustained", FALLBACK_PEAKS["bf16_tflops_sustained"])
    traffic = None
    tf = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tf):
        with open(tf) as f:
            traffic = json.load(f).get(f"cfg{cfg}", {}).get(dom)
    total_flops = sum(op_flops(k, B, T, C, NH) for k in totals if op_flops(k, B, T, C, NH))
    line = dict(
        metric="causal attention fwd+bwd tokens/sec", value=value, unit="tokens/s", n_gpus=world,
        steps=steps, warmup=warmup, ms_per_step=ms, higher_is_better=True, scaling="strong",
        vs_baseline=None, dtype="bf16" if w["prec"] == "bf16" else "f32", data="synthetic",
        config=dict(workload=w["name"], global_batch=GB, seq_len=T, d_model=C, heads=NH, head_dim=C // NH,
                    per_gpu_batch=B, parallelism=f"dp{world}", l2="inputs larger than L2 (no flush)"),
        roofline=dict(bound="tensor", kernel=dom, achieved=achieved, peak=peak, unit="TFLOP/s",
                      frac=achieved / peak, traffic=traffic,
                      peak_source=f"{src} bf16_tflops_sustained"),
        step_tflops=total_flops / (ms * 1e-3) / 1e12 if world == 1 else None,
        breakdown=per_op,
        gpu_launches=launches,
        e2e=dict(value=GB * T / (e2e_ms * 1e-3), unit="tokens/s", h2d_bytes_per_step=h2d * world,
                 d2h_bytes_per_step=d2h * world, ms_per_step=e2e_ms),
        clocks=clk,
    )
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg)
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", type=int, default=5, choices=sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="override the global batch (small cases for profiler captures only)")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args, args.config)
    return run_ours(args, args.config)


if __name__ == "__main__":
    sys.exit(main())
