"""Pins the C restatement (oracle/hmoe_oracle.c) before it is trusted.

Expected values come from tests/golden/*.npz, produced by the reference's own
CPU classes (tests/golden/make_golden.py), and from literal known answers in
the reference's tests.  The restatement must match bit for bit: it performs
the same floating-point operations in the same order.
"""
import hashlib

import numpy as np
import pytest

import hmoe_api as H
import oracle as O
from conftest import host_layer


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


@pytest.fixture(scope="module")
def port():
    return O.port()


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_router_matches_reference_fixture(port, golden, case):
    g = golden("router.npz")
    T, Hd, E, k, sm, rn, has_bias = (int(v) for v in g[f"{case}_cfg"])
    bias = g[f"{case}_bias"] if has_bias else None
    ids, sc, off, gt, gs = O.route(port, g[f"{case}_x"], g[f"{case}_w"], bias, k, bool(sm), bool(rn))
    np.testing.assert_array_equal(ids, g[f"{case}_ids"])
    np.testing.assert_array_equal(sc, g[f"{case}_scores"])
    np.testing.assert_array_equal(off, g[f"{case}_offsets"])
    np.testing.assert_array_equal(gt, g[f"{case}_gtok"])
    np.testing.assert_array_equal(gs, g[f"{case}_gsc"])


def test_phase12_grouping_known_answer(port, golden):
    # tests/phase12_tests.cpp:264-270: groups {0,2}, {0,1,2}, {1}.
    g = golden("router.npz")
    ids, sc, off, gt, gs = O.route(port, g["p12_x"], g["p12_w"], None, 2, True, True)
    groups = [list(gt[off[e]:off[e + 1]]) for e in range(3)]
    assert groups == [[0, 2], [0, 1, 2], [1]]
    np.testing.assert_array_equal(ids, g["p12_ids"])
    np.testing.assert_array_equal(sc, g["p12_scores"])
    # renormalised top-2 scores sum to 1 per token
    np.testing.assert_allclose(sc.sum(axis=1), 1.0, rtol=1e-6)


def test_phase18_router_known_answer(port, golden):
    g = golden("router.npz")
    ids, sc, *_ = O.route(port, g["p18_x"], g["p18_w"], None, 2, True, True)
    np.testing.assert_array_equal(ids, g["p18_ids"])
    np.testing.assert_array_equal(sc, g["p18_scores"])


def test_int8_gemm_matches_reference_and_double_oracle(port, golden):
    g = golden("int8_gemm_phase23.npz")
    import sys
    sys.path.insert(0, __file__.rsplit("/", 1)[0] + "/golden")
    from make_golden import GEMM_SHAPES, phase23_inputs
    for (r, k, n) in GEMM_SHAPES:
        x, q = phase23_inputs(r, k, n)
        out = O.int8_matmul(port, x, q, np.float32(0.003), -3)
        np.testing.assert_array_equal(out, g[f"out_{r}_{k}_{n}"])
        # independent double accumulation, tests/phase23_tests.cpp:232-240
        w = ((q.astype(np.int32) + 3).astype(np.float32) * np.float32(0.003)).astype(np.float64)
        ref = x.astype(np.float64) @ w
        assert np.all(np.abs(out - ref) <= 1e-5 + 1e-5 * np.abs(out))


def test_int8_mlp_matches_reference(port, golden):
    g = golden("int8_mlp_phase23.npz")

    def qmat(rows, cols):
        j = np.arange(rows * cols)
        return (((j * 13) % 255) - 127).astype(np.int8).reshape(rows, cols)

    y = O.expert_mlp(port, g["x"], qmat(513, 67), qmat(513, 67), qmat(67, 513),
                     np.full(3, 0.001, np.float32), np.zeros(3, np.int32))
    np.testing.assert_array_equal(y, g["y"])


def test_quantizer_matches_reference(port, golden):
    g = golden("quantize.npz")
    q, s, z, e = O.quantize(port, g["vals"])
    np.testing.assert_array_equal(q, g["q"])
    assert s == g["scale"] and z == g["zp"] == 0 and e == g["err"]
    assert e <= s * 0.5001  # tests/phase22_tests.cpp:171-174
    q2, s2, z2, e2 = O.quantize(port, g["w"])
    np.testing.assert_array_equal(q2, g["q2"])
    assert s2 == g["scale2"] and e2 == g["err2"]
    # the product-side packer (hmoe_quantize_int8) restates the same function
    q3, s3, z3, e3 = H.quantize_int8(g["w"])
    np.testing.assert_array_equal(q3, g["q2"])
    assert s3 == g["scale2"] and z3 == 0 and e3 == g["err2"]


@pytest.mark.parametrize("name,cfg,T,seed", [("c1_t64", "c1", 64, 0), ("c3_t16", "c3", 16, 0),
                                              ("c2_t3", "c2", 3, 1), ("c5_t4", "c5", 4, 2)])
def test_layer_matches_reference_fixture(port, golden, name, cfg, T, seed):
    g = golden(f"layer_{name}.npz")
    hl = host_layer(cfg, seed)
    x = H.make_tokens(H.CONFIGS[cfg], T, seed=seed)
    # the regenerated inputs are the ones the fixture was made from
    assert sha(x) == str(g["sha_x"])
    assert sha(hl.router_w) == str(g["sha_router"])
    assert sha(hl.arena) == str(g["sha_arena"])
    np.testing.assert_array_equal(hl.scales, g["scales"])
    out, ids, sc, off = O.moe_layer_port(hl, x)
    np.testing.assert_array_equal(ids, g["ids"])
    np.testing.assert_array_equal(sc, g["scores"])
    np.testing.assert_array_equal(off, g["offsets"])
    np.testing.assert_array_equal(out, g["out"])


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not built here")
@pytest.mark.parametrize("seed", [3, 4])
def test_port_matches_reference_on_random_layers(port, seed):
    cfg = H.LayerConfig(128, 192, 16, 4, True, seed % 2 == 0, 1, 1.1)
    hl = H.make_host_layer(cfg, seed=seed)
    x = H.make_tokens(cfg, 37, seed=seed)
    out_p, ids_p, sc_p, off_p = O.moe_layer_port(hl, x)
    out_r, ids_r, sc_r, off_r = O.RefLayer(hl).forward(x, threads=2, want_routing=True)
    np.testing.assert_array_equal(ids_p, ids_r)
    np.testing.assert_array_equal(sc_p, sc_r)
    np.testing.assert_array_equal(off_p, off_r)
    np.testing.assert_array_equal(out_p, out_r)


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not built here")
@pytest.mark.parametrize("T,Hd,eps", [(9, 2048, 1e-6), (4, 7, 1e-5), (2, 4096, 1e-6)])
def test_rms_norm_port_matches_reference(port, T, Hd, eps):
    """The port's RMSNorm equals the reference's own RMSNorm class on its CPU
    backend (src/transformer/norm/RMSNorm.cpp:64-77) bit for bit."""
    rng = np.random.default_rng(Hd)
    x = (rng.standard_normal((T, Hd)) * rng.uniform(1e-3, 1e3, size=(T, 1))).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(Hd)).astype(np.float32)
    np.testing.assert_array_equal(O.rms_norm_port(x, g, eps), O.rms_norm_ref(x, g, eps))


@pytest.mark.skipif(not O.ref_available(), reason="reference sources not built here")
def test_stack_port_matches_reference(port):
    """A stack of blocks with per-layer weights from (seed, layer): the
    post-attention RMSNorm, the MoE layer and the residual add of
    TransformerBlock::execute with an identity attention
    (src/transformer/runtime/TransformerBlock.cpp:90-104).  The port and the
    reference's own classes agree bit for bit through every block, routing
    included, and the residual stream stays finite."""
    cfg = H.LayerConfig(128, 192, 16, 4, True, True, 0, 1.1)
    xp = H.make_tokens(cfg, 19, seed=8)
    xr = xp.copy()
    for l in range(6):
        hl = H.make_host_layer(cfg, seed=8, layer=l)
        g = H.make_norm_weight(cfg, 8, l)
        out_p, ids_p, _, _ = O.moe_layer_port(hl, O.rms_norm_port(xp, g, 1e-6))
        out_r, ids_r, _, _ = O.RefLayer(hl).forward(O.rms_norm_ref(xr, g, 1e-6), threads=2, want_routing=True)
        np.testing.assert_array_equal(ids_p, ids_r)
        xp = (xp + out_p).astype(np.float32)
        xr = (xr + out_r).astype(np.float32)
        np.testing.assert_array_equal(xp, xr)
    assert np.isfinite(xp).all()


def test_router_rejects_non_finite(port):
    x = np.ones((2, 4), np.float32)
    w = np.ones((4, 3), np.float32)
    w[0, 0] = np.inf
    with pytest.raises(O.OracleError):
        O.route(port, x, w, None, 2)
