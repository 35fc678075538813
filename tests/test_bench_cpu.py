"""bench.py's reference arm on the host cores: the JSON line's contract, and the non-zero ranks.

The reference arm times the reference's own CPU path (restated by the oracle) and needs no GPU, so
its line can be checked here: the keys the driver reads, impl, a cpu_baseline describing the run,
and an e2e with no host<->device bytes.  Under torchrun only rank 0 prints.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(args, env_extra=None):
    env = dict(os.environ)
    env.update(env_extra or {})
    return subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT, env=env,
                          capture_output=True, text=True, timeout=300)


@pytest.mark.parametrize("config,metric", [(1, "causal attention fwd+bwd tokens/sec"),
                                           (4, "causal attention decode tokens/sec")])
def test_reference_arm_line(config, metric):
    r = _run(["--impl", "reference", "--config", str(config), "--steps", "2", "--warmup", "1"])
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == metric and d["unit"] == "tokens/s"
    assert d["value"] > 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["steps"] == 2 and d["warmup"] == 1 and d["data"] == "synthetic"
    assert d["vs_baseline"] is None and "workload" in d["config"]
    cb = d["cpu_baseline"]
    assert cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"] and cb["value"] > 0
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["e2e"]["value"] == d["value"]


def test_reference_arm_silent_on_other_ranks():
    r = _run(["--impl", "reference", "--config", "1", "--steps", "1", "--warmup", "0"], {"RANK": "1"})
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [ln for ln in r.stdout.splitlines() if ln.startswith("{")]


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench_under_test", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_roofline_accounting():
    """The FLOP counts behind every roofline fraction of the line: attention 4*D (forward) and 8*D
    (backward) per causal (query, key) pair, GEMMs 2*M*N*K, no credit for recomputing S; the
    attention-core and projection groups are sums over their own timed ranges."""
    b = _bench_module()
    B, T, C, NH = 512, 512, 768, 12
    D, M = C // NH, B * T
    pairs = B * NH * T * (T + 1) // 2
    assert b.op_flops("attn_fwd", B, T, C, NH) == 4 * D * pairs
    assert b.op_flops("attn_bwd", B, T, C, NH) == 8 * D * pairs
    assert b.op_flops("attn_bwd", B, T, C, NH) == pytest.approx(4.131e11, rel=1e-3)  # cfg 5, per step
    assert b.op_flops("gemm_qkv", B, T, C, NH) == 2 * M * 3 * C * C
    assert b.op_flops("gemm_dwqkv", B, T, C, NH) == b.op_flops("gemm_dx", B, T, C, NH)
    six = sum(b.op_flops(k, B, T, C, NH) for k in ("gemm_qkv", "gemm_out", "gemm_dwo", "gemm_dctx", "gemm_dwqkv",
                                                  "gemm_dx"))
    assert six == 24 * M * C * C
    assert b.op_flops("cast", B, T, C, NH) is None
    totals = {"attn_fwd": (0.5, 1), "attn_bwd": (1.5, 1), "gemm_qkv": (0.8, 1), "cast": (0.2, 1)}
    g = b.group_tflops(totals, lambda k: b.op_flops(k, B, T, C, NH))
    core = (12 * D * pairs) / 1e12
    assert g["attention_core"]["tflop_per_step"] == pytest.approx(core)
    assert g["attention_core"]["tflops"] == pytest.approx(core / 2.0e-3)
    assert g["projections"]["ms_per_step"] == pytest.approx(0.8)
    assert g["sum"]["ms_per_step"] == pytest.approx(2.8)  # the cast has no FLOPs and is left out
    peak, src, bound = b.precision_peak("tf32", {"bf16_tflops": 1635.0}, "measured")
    assert peak == pytest.approx(817.5) and bound == "tensor"
