"""The C-ABI library loads, exports every declared entry point, and its
host-only logic (planner, argument validation, synthetic inputs) behaves as
the reference does.  No GPU is touched here."""
import ctypes
import os
import re

import numpy as np
import pytest

import hmoe_api as H
from conftest import host_layer

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "hmoe.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(hmoe_[a-z0-9_]+)\s*\(", text)))


def test_header_and_exports_agree():
    assert declared_functions() == sorted(H.EXPORTS)
    lib = H.lib()
    for name in declared_functions():
        assert hasattr(lib, name), name


def test_library_is_built_for_sm100a():
    # the fatbin carries sm_100a code (checked through the loader, not by
    # disassembly): the build recipe is the only one in the tree.
    mk = open(os.path.join(ROOT, "hypermoe-engine_b200", "Makefile")).read()
    assert "arch=compute_100a,code=sm_100a" in mk


def plan(rows, inner, cols, mode=0):
    p = H.GemmPlan()
    rc = H.lib().hmoe_int8_gemm_plan(rows, inner, cols, mode, ctypes.byref(p))
    return rc, p


def test_planner_matches_reference_known_answers():
    # tests/phase23_tests.cpp:34-49
    rc, gate = plan(1, 2048, 768)
    assert rc == 0 and gate.implementation == 2 and gate.partitions == 4
    assert gate.blocks == 96 and gate.scratch_elements == 3072
    rc, down = plan(1, 768, 2048)
    assert down.partitions == 2 and down.blocks == 128
    assert plan(1, 2048, 768, 1)[1].blocks == 3
    assert plan(1, 8, 8)[1].implementation == 1
    assert plan(2, 257, 65)[1].scratch_elements == 0
    assert plan(1, 8193, 65)[1].partitions == 8
    assert plan(0, 10, 10)[0] == 1
    assert plan(2, (1 << 64) - 1, 2)[0] == 1
    assert plan(1, 1, 1, 99)[0] == 1


def test_cooperative_rejects_partition_mismatch_without_gpu():
    # CudaKernels.cu:330-333: wrong partition count -> invalid_argument,
    # decided on the host before any launch.
    L = H.lib()
    rc = L.hmoe_int8_weight_matmul_cooperative(1, 1, 1, 1, 1, 2048, 768, 3, 0.01, 0, None)
    assert rc == 1
    rc = L.hmoe_int8_weight_matmul_cooperative(1, 1, 1, None, 1, 2048, 768, 4, 0.01, 0, None)
    assert rc == 1


def test_invalid_layer_descriptors_rejected_on_host():
    d = H.LayerDesc()
    n = ctypes.c_size_t()
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 1
    cfg = H.CONFIGS["c3"]
    d.hidden, d.intermediate, d.experts, d.top_k = cfg.hidden, cfg.intermediate, cfg.experts, 9999
    d.router_weight = d.arena = d.quant = 256
    d.expert_stride = cfg.expert_stride
    d.ep_size = 1
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 1  # top_k > E
    d.top_k = 8
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4096, ctypes.byref(n)) == 0
    assert n.value > 4096 * 8 * (cfg.hidden * 4)
    d.hidden = 100  # not a multiple of 64
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 7
    d.hidden = cfg.hidden
    d.expert_stride = cfg.expert_stride + 8  # TMA needs 16-byte strides
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 1
    d.expert_stride = cfg.expert_stride
    # bulk/tensor copies and 16-byte vector accesses fault on misaligned
    # addresses: the layer's buffers are checked before anything is enqueued
    for field, bad in (("router_weight", 256 + 4), ("arena", 256 + 8), ("quant", 256 + 2), ("router_bias", 258)):
        setattr(d, field, bad)
        assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 1, field
        setattr(d, field, 256 if field != "router_bias" else None)
    assert H.lib().hmoe_workspace_size(ctypes.byref(d), 4, ctypes.byref(n)) == 0
    L = H.lib()
    for x, y, ws in ((4096 + 4, 8192, 1 << 20), (4096, 8192 + 8, 1 << 20), (4096, 8192, (1 << 20) + 4)):
        assert L.hmoe_moe_forward(ctypes.byref(d), x, y, 4, ws, 1 << 40, None) == 1
    assert L.hmoe_moe_forward_residual(ctypes.byref(d), 4096, 4096 + 12, 8192, None, 4, 1 << 20, 1 << 40, None) == 1
    assert L.hmoe_moe_forward_residual(ctypes.byref(d), 4096, None, 8192, 8192 + 2, 4, 1 << 20, 1 << 40, None) == 1
    assert L.hmoe_route(ctypes.byref(d), 4096 + 4, 4, None, None, None, None, None, 1 << 20, 1 << 40, None) == 1
    assert L.hmoe_moe_forward_host(ctypes.byref(d), 4096, 8192, 4, (1 << 20) + 8, 1 << 40, None) == 1


def test_synth_is_deterministic_across_thread_counts():
    a = H.synth_normal(5, 9, 0.02, (1000, 37), threads=1)
    b = H.synth_normal(5, 9, 0.02, (1000, 37), threads=7)
    np.testing.assert_array_equal(a, b)
    assert abs(float(a.std()) - 0.02) < 1e-3 and abs(float(a.mean())) < 1e-3
    c = H.synth_normal(5, 10, 0.02, (1000, 37), threads=3)
    assert not np.array_equal(a, c)


def test_zipf_bias_is_a_permuted_harmonic_prior():
    b = H.synth_zipf_bias(0, 1.1, 128)
    ranks = np.rint(np.exp(-b / 1.1) - 1).astype(int)
    assert sorted(ranks.tolist()) == list(range(128))
    assert b.max() == 0.0


def test_arena_layout_matches_packer():
    cfg = H.LayerConfig(64, 128, 3, 2, shared_experts=1)
    hl = H.make_host_layer(cfg, seed=1)
    assert hl.arena.size == 4 * cfg.expert_stride and cfg.expert_stride % 4096 == 0
    for e in range(4):
        for p in range(3):
            q = hl.arena[e * cfg.expert_stride + p * cfg.proj_bytes:][:cfg.proj_bytes]
            assert np.abs(q).max() == 127  # symmetric per-projection scale
            assert hl.zps[e, p] == 0 and hl.scales[e, p] > 0


def test_layer_binding_refuses_tensors_the_kernels_would_misread():
    """The ctypes layer methods hand raw pointers to the C ABI, so they
    refuse a token or output tensor of the wrong dtype, shape, layout or
    device before anything is enqueued (checked here without a GPU: every
    call below is refused on the host)."""
    import torch
    cfg = H.CONFIGS["c1"]
    dl = H.DeviceLayer(host_layer("c1", 0), "cpu")
    good = torch.zeros((4, cfg.hidden), dtype=torch.float32)
    bad_inputs = [good.double(), good.t().contiguous().t(), torch.zeros((4, cfg.hidden + 1)),
                  torch.zeros((4, cfg.hidden), dtype=torch.float32).view(2, 2 * cfg.hidden)]
    for x in bad_inputs:
        with pytest.raises(ValueError):
            dl.forward(x)
        with pytest.raises(ValueError):
            dl.route(x)
    with pytest.raises(ValueError):
        dl.forward(good, y=torch.zeros((3, cfg.hidden)))
    with pytest.raises(ValueError):
        dl.forward_residual(good, residual=good.half())
    with pytest.raises(ValueError):
        dl.forward_residual(good, y_bf16=torch.zeros((4, cfg.hidden), dtype=torch.float16))
    with pytest.raises(ValueError):
        dl.forward_host(good.double(), good)
