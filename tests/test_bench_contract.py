"""bench.py's reference arm (the reference's own CPU path, no GPU) keeps the
JSON contract the harness reads: one line with the metric, value, unit and
config of the product arm's line, an `impl` of "reference", a cpu_baseline
describing the run, and an e2e object with no host copies."""
import json
import os
import subprocess
import sys

import pytest

import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run(*args):
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", *args],
                       capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert p.returncode == 0, p.stderr[-2000:]
    lines = [ln for ln in p.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, p.stdout
    return json.loads(lines[0])


def _check_common(d):
    for key in ("metric", "value", "unit", "n_gpus", "steps", "ms_per_step", "higher_is_better", "scaling",
                "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["cpu_baseline"]["value"] == d["value"]
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["e2e"] == {"value": d["value"], "unit": d["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not built here")
def test_reference_arm_layer_line():
    d = _run("--steps", "1", "--warmup", "0", "--tokens", "16")
    _check_common(d)
    assert d["metric"] == "MoE-layer tokens/s (Qwen3-30B-A3B shape, INT8 experts)"
    assert d["config"]["workload"].startswith("c3") and d["config"]["tokens_per_gpu"] == 16
    assert d["single_thread"]["cores"] == 1 and d["single_thread"]["value"] > 0


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not built here")
def test_reference_arm_stack_line():
    d = _run("--config", "c4", "--layers", "2", "--steps", "2", "--stack-cpu-tokens", "2")
    _check_common(d)
    assert d["metric"] == "MoE-stack tokens/s (Qwen3-30B-A3B, 2 INT8 MoE layers)"
    assert d["config"]["layers"] == 2 and d["steps"] == 2
