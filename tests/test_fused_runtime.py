"""FusedMoERuntime (hypermoe-engine_b200/host/FusedMoERuntime.cpp): the
reference's layer-runtime contract (MoERuntime::executeBatch /
executeLayer, src/core/runtime/MoERuntime.hpp:28-60) over the fused sm_100a
layer, compiled against the reference's headers and driven through the
reference's own CudaTensorBackend by oracle/_ref/fused_runtime_check, which
compares it with the reference's CPU classes: ids and expert groups bit for
bit, scores to the CPU expf's last place, outputs within the INT8 layer
tolerance (tests/tolerance.py).  Without shared experts it also builds the
runtime from a packed ExpertStore written by the reference's own
ExpertStore::create (FusedMoERuntime::fromPackedStore: same output bit for
bit), runs the transformer block's MoE stage with the residual fused
(executeWithResidual: residual + output in one FP32 rounding, and its BF16
copy rounded to nearest even) and checks the all-resident budget rule."""
import json
import os
import subprocess

import pytest

import hmoe_api as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXE = os.path.join(ROOT, "oracle", "_ref", "fused_runtime_check")

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("cfg_name,T,seed", [("c1", 64, 0), ("c3", 16, 1), ("c3", 300, 2), ("c2", 3, 3)])
def test_fused_runtime_matches_reference_cpu_path(cuda, cfg_name, T, seed):
    if not os.path.exists(EXE):
        pytest.fail(f"{EXE} is not built (oracle/Makefile reftests, needs the reference sources)")
    c = H.CONFIGS[cfg_name]
    cmd = [EXE, "--hidden", str(c.hidden), "--inter", str(c.intermediate), "--experts", str(c.experts),
           "--topk", str(c.top_k), "--softmax", str(int(c.softmax)), "--renorm", str(int(c.renormalize)),
           "--shared", str(c.shared_experts), "--zipf", str(c.zipf_alpha or 0), "--tokens", str(T),
           "--seed", str(seed)]
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert p.returncode == 0, (p.stdout + p.stderr)[-3000:]
    r = json.loads(p.stdout.strip().splitlines()[-1])
    assert r["ok"] and r["ids_equal"] and r["groups_equal"] and r["execute_layer_ok"], r
    # all-resident mode from a packed ExpertStore, the fused residual stage
    # and the budget rule (configurations without shared experts)
    assert r["packed_store_ok"] and r["residual_ok"] and r["covers_ok"], r
