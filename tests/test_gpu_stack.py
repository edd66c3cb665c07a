"""Stacks of MoE blocks (BASELINE's 48-layer Qwen3-30B-A3B configuration, at
test sizes) through the C ABI.  Every block is hmoe_rms_norm followed by
hmoe_moe_forward_residual (hmoe_ep_moe_forward_residual under expert
parallelism) applied in place, x_{l+1} = x_l + layer_l(rms_norm(x_l) * g_l),
as TransformerBlock::execute does with an identity attention
(src/transformer/runtime/TransformerBlock.cpp:90-104).

Parity is checked layer by layer on the device's own layer inputs: a stack's
output drifts from a CPU stack within the tolerance, so a CPU stack fed its
own activations could route a near-tied token differently at a later layer.
Each normalised input the device produced is compared with the reference's
own RMSNorm of the device's residual input, routed by the oracle (ids
bit-exact) and run through the oracle's layer (within the layer
tolerance); the next residual input must equal the previous one plus the
plain layer output (hmoe_moe_forward) bit for bit."""
import os
import sys
from datetime import timedelta

import numpy as np
import pytest

import hmoe_api as H
import oracle as O
from tolerance import assert_layer_close

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATHS = [os.path.join(ROOT, "hypermoe-engine_b200"), os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")]


def _hosts(cfg, n, seed):
    return [H.make_host_layer(cfg, seed=seed, layer=l) for l in range(n)]


def _assert_within_one_ulp(a, b):
    """Device RMSNorm against the reference's: the square sums are taken in
    double in a different order, which moves a float result by at most one
    unit in the last place (and almost never at all)."""
    assert a.shape == b.shape
    diff = np.abs(a.astype(np.float64) - b.astype(np.float64))
    assert (diff <= np.spacing(np.abs(b)).astype(np.float64)).all(), float(diff.max())
    assert np.mean(a == b) > 0.999


@pytest.mark.parametrize("T,Hd,eps,scale", [(5, 2048, 1e-6, 1.0), (3, 7, 1e-6, 1.0), (17, 4096, 1e-5, 300.0),
                                            (64, 256, 1e-6, 1e-3)])
def test_rms_norm_matches_reference(cuda, T, Hd, eps, scale):
    """hmoe_rms_norm against the reference's own RMSNorm class on its CPU
    backend (RMSNorm.cpp:64-77), vectorised (H % 4 == 0) and scalar rows,
    in place, and the argument checks of RMSNorm's constructor."""
    import torch
    rng = np.random.default_rng(T + Hd)
    x = (rng.standard_normal((T, Hd)) * scale * rng.uniform(0.1, 10.0, size=(T, 1))).astype(np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(Hd)).astype(np.float32)
    ref = O.rms_norm_ref(x, g, eps)
    np.testing.assert_array_equal(O.rms_norm_port(x, g, eps), ref)  # the port is pinned to it
    dx, dg = torch.from_numpy(x).to(cuda), torch.from_numpy(g).to(cuda)
    out = H.rms_norm(dx, dg, eps=eps)
    _assert_within_one_ulp(out.cpu().numpy(), ref)
    H.rms_norm(dx, dg, out=dx, eps=eps)  # in place
    np.testing.assert_array_equal(dx.cpu().numpy(), out.cpu().numpy())
    L = H.lib()
    assert L.hmoe_rms_norm(dx.data_ptr(), dg.data_ptr(), out.data_ptr(), T, Hd, 0.0, None) == 1
    assert L.hmoe_rms_norm(dx.data_ptr(), dg.data_ptr(), out.data_ptr(), T, Hd, float("nan"), None) == 1
    assert L.hmoe_rms_norm(dx.data_ptr(), None, out.data_ptr(), T, Hd, eps, None) == 1
    assert L.hmoe_rms_norm(None, None, None, 0, Hd, eps, None) == 0
    torch.cuda.synchronize()


@pytest.mark.parametrize("cfg_name,n_layers,T", [("c1", 4, 64), ("c3", 3, 24), ("c2", 2, 5)])
def test_stack_layers_match_oracle(cuda, cfg_name, n_layers, T):
    import torch
    cfg = H.CONFIGS[cfg_name]
    hosts = _hosts(cfg, n_layers, seed=21)
    # per-layer weights come from (seed, layer): the layers differ
    assert not np.array_equal(hosts[0].arena, hosts[1].arena)
    assert not np.array_equal(hosts[0].router_w, hosts[1].router_w)
    stack = H.MoEStack(cfg, n_layers, seed=21, device=cuda, hosts=hosts)
    assert not np.array_equal(stack.norm_host[0], stack.norm_host[1])
    x_np = H.make_tokens(cfg, T, seed=21)
    x = torch.from_numpy(x_np).to(cuda)
    trace = []
    stack.forward(x, trace=trace)
    torch.cuda.synchronize()
    assert stack.read_status()[0] == 0
    assert len(trace) == n_layers
    xs = [r for r, _ in trace] + [x.cpu().numpy()]
    np.testing.assert_array_equal(xs[0], x_np)
    for l, layer in enumerate(stack.layers):
        xn = trace[l][1]
        _assert_within_one_ulp(xn, O.rms_norm_ref(xs[l], stack.norm_host[l], stack.eps))
        dxn = torch.from_numpy(xn).to(cuda)
        plain = layer.forward(dxn).cpu().numpy()
        ids, *_ = layer.route(dxn)
        np.testing.assert_array_equal(xs[l + 1], (xs[l] + plain).astype(np.float32))
        out_p, ids_p, _, _ = O.moe_layer_port(hosts[l], xn)
        assert np.array_equal(ids.cpu().numpy().view(np.uint32), ids_p), f"layer {l}: routing differs"
        assert_layer_close(xs[l + 1].astype(np.float64) - xs[l].astype(np.float64), out_p)
        assert layer.read_status()[0] == 0, l
    assert np.isfinite(xs[-1]).all()


@pytest.mark.parametrize("peer", [True, False])
@pytest.mark.parametrize("cfg_name,n_layers,T", [("c1", 3, 40), ("c3", 2, 200)])
def test_stack_ep_one_rank_equals_single_gpu(cuda, cfg_name, n_layers, T, peer):
    """The expert-parallel stack (one communicator, one registered workspace
    shared by every layer, hmoe_ep_moe_forward_residual per layer) on a
    one-rank communicator equals the single-GPU stack bit for bit for the
    tensor-core variant."""
    import torch
    cfg = H.CONFIGS[cfg_name]
    hosts = _hosts(cfg, n_layers, seed=22)
    x_np = H.make_tokens(cfg, T, seed=22)
    H.set_variant(2)
    comm = H.EpComm(H.ep_unique_id(), 0, 1, timeout_ms=30000)
    try:
        ref = H.MoEStack(cfg, n_layers, seed=22, device=cuda, hosts=hosts)
        y_ref = ref.forward(torch.from_numpy(x_np).to(cuda)).cpu().numpy()
        del ref
        ep = H.MoEStack(cfg, n_layers, seed=22, device=cuda, comm=comm, peer=peer, hosts=hosts)
        x = torch.from_numpy(x_np).to(cuda)
        y1 = ep.forward(x, max_tokens=T + 3).cpu().numpy()
        st = ep.read_status()[0]
        y2 = ep.forward(torch.from_numpy(x_np).to(cuda), max_tokens=T + 3).cpu().numpy()
        ws_ptrs = {layer._ws.data_ptr() for layer in ep.layers}
    finally:
        H.set_variant(0)
        comm.close()
    assert st == 0
    assert len(ws_ptrs) == 1  # one workspace for the whole stack
    np.testing.assert_array_equal(y1, y_ref)
    np.testing.assert_array_equal(y2, y_ref)


def _stack_rank(rank, P, port, cfg_name, n_layers, Ts, q):
    for p in PATHS:
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import hmoe_api as H

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=P, timeout=timedelta(seconds=120))
    comm = None
    try:
        obj = [H.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = H.EpComm(obj[0], rank, P, timeout_ms=60000)
        cfg = H.CONFIGS[cfg_name]
        x_all = H.make_tokens(cfg, sum(Ts), seed=23)
        t0 = sum(Ts[:rank])
        dev = torch.device("cuda", rank)
        H.set_variant(2)
        stack = H.MoEStack(cfg, n_layers, seed=23, device=dev, comm=comm)
        dx = torch.from_numpy(x_all[t0:t0 + Ts[rank]]).to(dev)
        y = stack.forward(dx, max_tokens=max(Ts)).cpu().numpy()
        st, _, _ = stack.read_status()
        q.put((rank, st, y))
    except Exception as exc:
        q.put((rank, -1, repr(exc)))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg_name,n_layers,Ts", [("c3", 3, (256, 100)), ("c3", 2, (64, 0, 200, 31))])
def test_stack_ep_ranks_equal_single_gpu(cuda, cfg_name, n_layers, Ts):
    """P = len(Ts) ranks, one process per GPU (skipped with fewer GPUs):
    the expert-parallel stack's slices equal the single-GPU stack on the
    concatenated batch bit for bit (tensor-core variant)."""
    import socket

    import torch
    import torch.multiprocessing as mp
    P = len(Ts)
    if torch.cuda.device_count() < P:
        pytest.skip(f"needs {P} GPUs")
    cfg = H.CONFIGS[cfg_name]
    x_all = H.make_tokens(cfg, sum(Ts), seed=23)
    H.set_variant(2)
    try:
        ref = H.MoEStack(cfg, n_layers, seed=23, device=cuda)
        y_ref = ref.forward(torch.from_numpy(x_all).to(cuda)).cpu().numpy()
        del ref
        torch.cuda.empty_cache()
    finally:
        H.set_variant(0)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_stack_rank, args=(r, P, port, cfg_name, n_layers, Ts, q)) for r in range(P)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(P):
            rank, st, y = q.get(timeout=600)
            out[rank] = (st, y)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(P):
        assert out[r][0] == 0, out[r][1]
    np.testing.assert_array_equal(np.concatenate([out[r][1] for r in range(P)]), y_ref)
