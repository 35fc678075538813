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
