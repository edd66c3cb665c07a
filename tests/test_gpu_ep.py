"""Expert parallelism on the GPU through the C ABI (hmoe_ep_*).

* One GPU: a communicator of one rank runs the whole EP path -- the
  peer-memory path (registered workspace: device count exchange and plan,
  row stores, epoch flags) and the NCCL path (count all-gather, host plan,
  send/recv to itself) -- through received-segment tiles, return and
  combine; its output must equal hmoe_moe_forward bit for bit.
* Two or more GPUs: two ranks, one process per GPU, each with its own
  slice of the batch and half of the experts; every rank's output must equal
  the single-GPU hmoe_moe_forward on the concatenated batch bit for bit
  (same expert-MLP variant, fixed combine order) and the oracle within the
  layer tolerance.
"""
import os
import socket
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
GEMV_MAX_ROWS = 8  # kGemvMaxAssignments (csrc/layer.cuh): larger launches take the GEMM


def _single_gpu(hl, x, dev, variant):
    import torch
    H.set_variant(variant)
    try:
        dl = H.DeviceLayer(hl, dev)
        y = dl.forward(torch.from_numpy(x).to(dev))
        torch.cuda.synchronize()
        return y.cpu().numpy()
    finally:
        H.set_variant(0)


@pytest.mark.parametrize("peer", [True, False])
@pytest.mark.parametrize("cfg_name,T,variant,placed", [("c3", 256, 0, False), ("c3", 256, 2, False),
                                                       ("c3", 1, 0, False), ("c2", 33, 2, False),
                                                       ("c1", 64, 1, False), ("c3", 256, 2, True),
                                                       ("c2", 33, 2, True)])
def test_ep_one_rank_equals_forward(cuda, cfg_name, T, variant, placed, peer):
    import torch
    cfg = H.CONFIGS[cfg_name]
    hl = H.make_host_layer(cfg, seed=3)
    x = H.make_tokens(cfg, T, seed=3)
    ref_variant = variant
    if variant == 0:
        # the automatic choice: the EP path decides by its row capacity
        # (peer path) or by the rows it received (NCCL path), the one-GPU
        # layer by its batch; compare against the variant the EP path takes
        rows = (T + 7) * cfg.top_k if peer else T * cfg.top_k
        ref_variant = 1 if rows <= GEMV_MAX_ROWS else 2
    ref = _single_gpu(hl, x, cuda, ref_variant)
    comm = H.EpComm(H.ep_unique_id(), 0, 1, timeout_ms=30000)
    try:
        H.set_variant(variant)
        # a scrambled placement: groups travel in slot order, rows still
        # combine in ascending expert id
        pl = np.random.default_rng(3).permutation(cfg.experts).astype(np.int32) if placed else None
        layer = H.EpLayer(hl, comm, cuda, slot_of_expert=pl, peer=peer)
        dx = torch.from_numpy(x).to(cuda)
        y1 = layer.forward(dx, max_tokens=T + 7).cpu().numpy()
        y2 = layer.forward(dx, max_tokens=T + 7).cpu().numpy()
        st, ties, _ = layer.read_status()
        plan = comm.last_plan()
        assert plan.recv_total == T * cfg.top_k
    finally:
        H.set_variant(0)
        comm.close()
    assert st == 0 and ties == 0
    assert np.array_equal(y1, y2)
    if variant != 1 or cfg.shared_experts == 0:
        assert np.array_equal(y1, ref), float(np.abs(y1 - ref).max())
    assert_layer_close(y1, O.moe_layer_port(hl, x)[0])


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_peer_flag_wait_times_out(cuda):
    """The peer path's flag wait is bounded: waiting for an epoch no rank
    reaches gives up after the limit, reports HMOE_TIMEOUT, and the context
    stays usable."""
    import torch
    cfg = H.CONFIGS["c1"]
    hl = H.make_host_layer(cfg, seed=1)
    comm = H.EpComm(H.ep_unique_id(), 0, 1, timeout_ms=30000)
    try:
        layer = H.EpLayer(hl, comm, cuda)
        x = torch.from_numpy(H.make_tokens(cfg, 8, seed=1)).to(cuda)
        layer.forward(x, max_tokens=8)
        assert comm.selftest_flag_wait(20_000_000) == 5  # HMOE_TIMEOUT
        y = layer.forward(x, max_tokens=8).cpu().numpy()  # still works
        assert layer.read_status()[0] == 0
        assert np.isfinite(y).all()
    finally:
        comm.close()


def _ep_rank(rank, P, port, cfg_name, Ts, variant, q, balanced=False, peer=True):
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
        hl = H.make_host_layer(cfg, seed=5)
        x_all = H.make_tokens(cfg, sum(Ts), seed=5)
        t0 = sum(Ts[:rank])
        dev = torch.device("cuda", rank)
        H.set_variant(variant)
        pl = None
        if balanced:  # placement from the router's popularity prior
            load = np.exp(hl.router_bias.astype(np.float64)) if hl.router_bias is not None else np.ones(cfg.experts)
            pl = H.ep_balanced_placement(load, P)
        layer = H.EpLayer(hl, comm, dev, slot_of_expert=pl, peer=peer)
        dx = torch.from_numpy(x_all[t0:t0 + Ts[rank]]).to(dev)
        y = layer.forward(dx, max_tokens=max(Ts)).cpu().numpy()
        y2 = layer.forward(dx, max_tokens=max(Ts)).cpu().numpy()  # a second epoch
        assert np.array_equal(y, y2)
        st, ties, _ = layer.read_status()
        q.put((rank, st, y))
    except Exception as exc:
        q.put((rank, -1, repr(exc)))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("cfg_name,Ts,variant,balanced,peer", [
    ("c3", (300, 212), 2, False, True),
    ("c2", (40, 0), 2, False, True),
    ("c3", (3, 1), 0, False, True),
    ("c3", (300, 212), 2, True, True),
    ("c3", (300, 212), 2, True, False),
    ("c3", (300, 212, 77, 0), 2, True, True),
    ("c2", (40, 0, 17, 3), 2, False, True),
    ("c3", (300, 212, 77, 0), 2, False, False),
    ("c3", (300, 212, 77, 0, 140, 5, 256, 31), 2, True, True),
    ("c3", (1, 2, 0, 1, 3, 1, 1, 2), 0, False, True),
    ("c3", (300, 212, 77, 0, 140, 5, 256, 31), 2, False, False),
])
def test_ep_ranks_equal_single_gpu(cuda, cfg_name, Ts, variant, balanced, peer):
    """P = len(Ts) ranks (one process per GPU, skipped with fewer GPUs): each
    rank's slice of the output equals the single-GPU layer on the
    concatenated batch (bit for bit for the tensor-core variant) and the
    oracle within the layer tolerance; ragged batches and empty ranks."""
    import torch
    import torch.multiprocessing as mp
    P = len(Ts)
    if torch.cuda.device_count() < P:
        pytest.skip(f"needs {P} GPUs")
    cfg = H.CONFIGS[cfg_name]
    hl = H.make_host_layer(cfg, seed=5)
    x_all = H.make_tokens(cfg, sum(Ts), seed=5)
    ref = _single_gpu(hl, x_all, cuda, variant)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, P, port, cfg_name, Ts, variant, q, balanced, peer))
             for r in range(P)]
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
    y = np.concatenate([out[r][1] for r in range(P)])
    if variant == 2:
        assert np.array_equal(y, ref), float(np.abs(y - ref).max())
    assert_layer_close(y, O.moe_layer_port(hl, x_all)[0])


def _ep_abort_rank(rank, port, q):
    """Rank 1 holds back while rank 0 runs a forward on the peer path, so
    rank 0's flag wait runs out; both then report the failure, and a fresh
    registration brings the path back."""
    for p in PATHS:
        sys.path.insert(0, p)
    import time

    import torch
    import torch.distributed as dist

    import hmoe_api as H

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=120))
    comm = None
    try:
        obj = [H.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        comm = H.EpComm(obj[0], rank, 2, timeout_ms=2000)  # flag waits give up after 2 s
        cfg = H.CONFIGS["c1"]
        hl = H.make_host_layer(cfg, seed=9)
        x_all = H.make_tokens(cfg, 24, seed=9)
        dev = torch.device("cuda", rank)
        layer = H.EpLayer(hl, comm, dev, peer=True)
        ws = layer.ep_workspace(16)  # collective registration
        dx = torch.from_numpy(x_all[rank * 12:(rank + 1) * 12]).to(dev)
        res = {}
        if rank == 0:
            t0 = time.perf_counter()
            layer.forward(dx, max_tokens=16)
            res["first"] = layer.read_status()[0]
            res["first_s"] = time.perf_counter() - t0
        dist.barrier()  # rank 0's wait has run out before rank 1 starts
        if rank == 1:
            t0 = time.perf_counter()
            layer.forward(dx, max_tokens=16)
            res["first"] = layer.read_status()[0]
            res["first_s"] = time.perf_counter() - t0
        dist.barrier()
        layer.forward(dx, max_tokens=16)  # still aborted: fails at the count exchange
        res["second"] = layer.read_status()[0]
        dist.barrier()
        comm.register_workspace(ws)  # collective: clears the abort mark
        y = layer.forward(dx, max_tokens=16).cpu().numpy()
        res["after"] = layer.read_status()[0]
        q.put((rank, res, y))
    except Exception as exc:
        q.put((rank, {"error": repr(exc)}, None))
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


def test_ep_peer_timeout_aborts_every_rank(cuda):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = H.CONFIGS["c1"]
    hl = H.make_host_layer(cfg, seed=9)
    x_all = H.make_tokens(cfg, 24, seed=9)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_abort_rank, args=(r, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, res, y = q.get(timeout=300)
            out[rank] = (res, y)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(2):
        res = out[r][0]
        assert "error" not in res, res
        assert res["first"] == 5 and res["second"] == 5 and res["after"] == 0, (r, res)
    assert 1.5 < out[0][0]["first_s"] < 30   # rank 0 waited out its limit
    assert out[1][0]["first_s"] < 1.5        # rank 1 failed at once
    y = np.concatenate([out[0][1], out[1][1]])
    assert_layer_close(y, O.moe_layer_port(hl, x_all)[0])
