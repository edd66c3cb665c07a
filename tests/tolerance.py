"""Output tolerances of the fused BF16 tensor-core path against the FP32
reference, and of the FP32 per-operator drop-ins.

* Layer outputs (BF16 operands, FP32 accumulation vs the reference's FP32
  CPU backend): the reference's own INT8 tolerance,
  CorrectnessOracle::toleranceFor(INT8) = {abs 2e-2, rel 2e-2}
  (src/validation/CorrectnessOracle.cpp:34-42), element-wise as in
  CorrectnessOracle::compare (:44-67); plus a normwise relative error
  <= 2e-2 and cosine similarity >= 0.9995 over the whole output.
* Per-operator FP32 drop-ins: |a - e| <= 1e-5 + 1e-5*|e|, the bound the
  reference's tests put on its own CUDA kernels (tests/phase23_tests.cpp:228).
"""
import numpy as np

LAYER_ABS = 2e-2
LAYER_REL = 2e-2
LAYER_NORMWISE = 2e-2
LAYER_COSINE = 0.9995
OP_ABS = 1e-5
OP_REL = 1e-5


def layer_report(actual, expected):
    a = np.asarray(actual, np.float64).ravel()
    e = np.asarray(expected, np.float64).ravel()
    diff = np.abs(a - e)
    elem_ok = bool(np.all(np.isfinite(a)) and np.all(diff <= LAYER_ABS + LAYER_REL * np.abs(e)))
    nrm = float(np.linalg.norm(a - e) / max(np.linalg.norm(e), 1e-30))
    cos = float(np.dot(a, e) / max(np.linalg.norm(a) * np.linalg.norm(e), 1e-30))
    return {"elementwise": elem_ok, "normwise": nrm, "cosine": cos, "max_abs": float(diff.max(initial=0.0))}


def assert_layer_close(actual, expected):
    r = layer_report(actual, expected)
    assert r["elementwise"], r
    assert r["normwise"] <= LAYER_NORMWISE, r
    assert r["cosine"] >= LAYER_COSINE, r
    return r


def assert_op_close(actual, expected):
    a = np.asarray(actual, np.float64)
    e = np.asarray(expected, np.float64)
    assert np.all(np.isfinite(a))
    bad = np.abs(a - e) > OP_ABS + OP_REL * np.abs(e)
    assert not bad.any(), (np.abs(a - e).max(), int(bad.sum()))
