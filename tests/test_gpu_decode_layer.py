"""The single-kernel decode layer (hypermoe-engine_b200/csrc/decode_layer.cu)
through the C ABI.  For batches of at most 2 tokens (8 when forced)
hmoe_moe_forward runs the whole layer as one cooperative kernel; its arithmetic, every summation order
included, is the multi-kernel GEMV variant's, so the two agree bit for bit,
and both match the reference-pinned port within the layer tolerance
(tests/tolerance.py).  Routing is the decode router's, certified against the
reference's sequential FP64 sum."""
import ctypes

import numpy as np
import pytest

import hmoe_api as H
import oracle as O
from conftest import host_layer
from tolerance import assert_layer_close

pytestmark = pytest.mark.gpu

DECODE = 3  # hmoe_set_variant: the decode layer only
GEMV = 1    # the multi-kernel GEMV variant
GEMM = 2    # the multi-kernel tensor-core GEMM variant


def t(a, dev):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).to(dev)


def host(x):
    import torch
    torch.cuda.synchronize()
    return x.cpu().numpy()


def forward_with(dl, x, variant, **kw):
    H.set_variant(variant)
    try:
        if kw:
            return host(dl.forward_residual(x, **kw))
        return host(dl.forward(x))
    finally:
        H.set_variant(0)


@pytest.mark.parametrize("cfg_name,T", [("c1", 1), ("c1", 8), ("c2", 1), ("c2", 3), ("c3", 1), ("c3", 2),
                                        ("c3", 5), ("c3", 8), ("c5", 1), ("c5", 8)])
def test_decode_layer_equals_gemv_variant(cuda, cfg_name, T):
    cfg = H.CONFIGS[cfg_name]
    hl = host_layer(cfg_name, 21)
    x_np = H.make_tokens(cfg, T, seed=21 + T)
    dl = H.DeviceLayer(hl, cuda)
    x = t(x_np, cuda)
    ref = forward_with(dl, x, GEMV)
    assert dl.read_status()[0] == 0
    y = forward_with(dl, x, DECODE)
    st, ties, _ = dl.read_status()
    assert st == 0 and ties == 0
    np.testing.assert_array_equal(y, ref)
    # the automatic choice: the decode layer up to 2 tokens, then the GEMV up
    # to 8 permuted rows, then the tensor-core GEMM
    rows = T * (cfg.top_k + cfg.shared_experts)
    auto = ref if T <= 2 or rows <= 8 else forward_with(dl, x, GEMM)
    np.testing.assert_array_equal(host(dl.forward(x)), auto)
    # and the port (the reference's CPU path restated, pinned bit for bit)
    out_p, *_ = O.moe_layer_port(hl, x_np)
    assert_layer_close(y, out_p)


@pytest.mark.parametrize("cfg_name,T", [("c1", 4), ("c3", 8)])
def test_decode_layer_residual_and_bf16(cuda, cfg_name, T):
    """The residual add and the BF16 copy fused into the decode layer's
    combine give what the multi-kernel combine gives, bit for bit."""
    import torch
    cfg = H.CONFIGS[cfg_name]
    hl = host_layer(cfg_name, 22)
    x = t(H.make_tokens(cfg, T, seed=22), cuda)
    res = t(H.make_tokens(cfg, T, seed=23), cuda)
    dl = H.DeviceLayer(hl, cuda)
    a16 = torch.empty((T, cfg.hidden), dtype=torch.bfloat16, device=cuda)
    b16 = torch.empty_like(a16)
    a = forward_with(dl, x, GEMV, residual=res, y_bf16=a16)
    b = forward_with(dl, x, DECODE, residual=res, y_bf16=b16)
    np.testing.assert_array_equal(a, b)
    assert torch.equal(a16, b16)
    assert dl.read_status()[0] == 0


def test_decode_layer_is_deterministic_and_graph_capturable(cuda):
    import torch
    cfg = H.CONFIGS["c3"]
    hl = host_layer("c3", 21)
    T = 4
    x = t(H.make_tokens(cfg, T, seed=24), cuda)
    dl = H.DeviceLayer(hl, cuda)
    y = torch.empty((T, cfg.hidden), device=cuda)
    first = host(dl.forward(x, y=y)).copy()
    np.testing.assert_array_equal(host(dl.forward(x, y=y)), first)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        dl.forward(x, y=y, stream=s)  # workspace allocated before the capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        dl.forward(x, y=y, stream=torch.cuda.current_stream())
    for _ in range(3):
        y.fill_(float("nan"))
        g.replay()
        np.testing.assert_array_equal(host(y), first)
    assert dl.read_status()[0] == 0


def test_decode_layer_reports_non_finite_router_input(cuda):
    cfg = H.CONFIGS["c3"]
    hl = host_layer("c3", 21)
    x = H.make_tokens(cfg, 3, seed=25)
    x[1, 7] = np.nan
    dl = H.DeviceLayer(hl, cuda)
    forward_with(dl, t(x, cuda), DECODE)
    assert dl.read_status()[0] == 2  # HMOE_NON_FINITE_ROUTER
    x[1, 7] = 0.0
    forward_with(dl, t(x, cuda), DECODE)
    assert dl.read_status()[0] == 0


def test_forced_decode_layer_rejects_larger_batches(cuda):
    import torch
    cfg = H.CONFIGS["c3"]
    dl = H.DeviceLayer(host_layer("c3", 21), cuda)
    T = 9
    x = torch.zeros((T, cfg.hidden), device=cuda)
    y = torch.zeros_like(x)
    ws = dl.workspace(T)
    H.set_variant(DECODE)
    try:
        rc = H.lib().hmoe_moe_forward(ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), T, ws.data_ptr(),
                                      ws.numel(), torch.cuda.current_stream().cuda_stream)
    finally:
        H.set_variant(0)
    assert rc == 7  # HMOE_UNSUPPORTED


@pytest.mark.parametrize("cfg_name,T", [("c3", 1), ("c3", 6), ("c1", 8)])
def test_decode_layer_exact_ties_break_by_expert_id(cuda, cfg_name, T):
    """Router columns duplicated (and, for C3, the bias made equal) give
    experts with identical logits for every token; both selections order
    them by ascending id (CpuRouterBackend.cpp:57-62), so the CTA-wide ranking
    of the decode layer and the warp rounds of the routers agree bit for
    bit, and exact ties are not counted as near-ties."""
    import dataclasses
    cfg = H.CONFIGS[cfg_name]
    base = host_layer(cfg_name, 21)
    w = base.router_w.copy()
    w[:, 1] = w[:, 0]
    w[:, 3] = w[:, 0]
    w[:, 6] = w[:, 2]
    bias = None
    if base.router_bias is not None:
        bias = base.router_bias.copy()
        bias[1] = bias[3] = bias[0]
        bias[6] = bias[2]
        # make the tied experts win often
        bias[0] = bias[2] = float(bias.max()) + 1.0
        bias[1] = bias[3] = bias[0]
        bias[6] = bias[2]
    hl = dataclasses.replace(base, router_w=w, router_bias=bias)
    x_np = H.make_tokens(cfg, T, seed=31)
    dl = H.DeviceLayer(hl, cuda)
    x = t(x_np, cuda)
    ref = forward_with(dl, x, GEMV)
    assert dl.read_status()[:2] == (0, 0)
    y = forward_with(dl, x, DECODE)
    assert dl.read_status()[:2] == (0, 0)
    np.testing.assert_array_equal(y, ref)
    out_p, *_ = O.moe_layer_port(hl, x_np)
    assert_layer_close(y, out_p)
