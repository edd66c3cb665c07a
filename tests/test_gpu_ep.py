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
    ref = _single_gpu(hl, x, cuda, variant)
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


@pytest.mark.parametrize("cfg_name,Ts,variant,balanced,peer", [("c3", (300, 212), 2, False, True),
                                                               ("c2", (40, 0), 2, False, True),
                                                               ("c3", (3, 1), 0, False, True),
                                                               ("c3", (300, 212), 2, True, True),
                                                               ("c3", (300, 212), 2, True, False)])
def test_ep_two_gpus_equal_single_gpu(cuda, cfg_name, Ts, variant, balanced, peer):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = H.CONFIGS[cfg_name]
    hl = H.make_host_layer(cfg, seed=5)
    x_all = H.make_tokens(cfg, sum(Ts), seed=5)
    ref = _single_gpu(hl, x_all, cuda, variant)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ep_rank, args=(r, 2, port, cfg_name, Ts, variant, q, balanced, peer))
             for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    try:
        for _ in range(2):
            rank, st, y = q.get(timeout=600)
            out[rank] = (st, y)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for r in range(2):
        assert out[r][0] == 0, out[r][1]
    y = np.concatenate([out[0][1], out[1][1]])
    if variant == 2:
        assert np.array_equal(y, ref), float(np.abs(y - ref).max())
    assert_layer_close(y, O.moe_layer_port(hl, x_all)[0])
