"""Expert-parallel protocols on CPU ranks (gloo), checked against the oracle.

Each rank routes its own tokens with the CPU oracle, all-gathers the
per-(rank, expert) row counts, plans its transfers with the library's
hmoe_ep_plan (the same host code hmoe_ep_moe_forward runs), ships rows and
routing weights to the expert owners, runs the owners' experts (oracle
expert MLP, local arena from local_host_layer), ships weighted outputs back
and combines in ascending expert id.  The result must equal the
single-process oracle layer (oracle/hmoe_oracle.c hmo_moe_layer, which
follows MoERuntime.cpp:58-349) on the concatenated batch bit for bit: the
protocol only moves rows, so any difference is a planning or ordering bug.

The *_peer_* tests restate the peer-memory path's layout instead (rows
stored into and read back from the owners' receive rows at indices derived
on every rank from the exchanged counts) and hold it to the same standard.
"""
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

import hmoe_api as H

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PATHS = [os.path.join(ROOT, "hypermoe-engine_b200"), os.path.join(ROOT, "oracle")]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _expert(hl, e):
    c = hl.cfg
    HI = c.proj_bytes
    blob = hl.arena[e * c.expert_stride:e * c.expert_stride + 3 * HI]
    return (blob[:HI].reshape(c.hidden, c.intermediate), blob[HI:2 * HI].reshape(c.hidden, c.intermediate),
            blob[2 * HI:].reshape(c.intermediate, c.hidden), hl.scales[e], hl.zps[e])


def _rank_main(rank, P, port, cfg_args, Ts, seed, q, placement=None):
    for p in PATHS:
        sys.path.insert(0, p)
    import torch
    import torch.distributed as dist

    import hmoe_api as H
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=P, timeout=timedelta(seconds=120))
    try:
        cfg = H.LayerConfig(*cfg_args)
        hl = H.make_host_layer(cfg, seed=seed, threads=1)
        local = H.local_host_layer(hl, P, rank, placement)
        # slot order of the expert groups (identity without a placement)
        expert_of_slot = (np.argsort(np.asarray(placement)) if placement is not None
                          else np.arange(cfg.experts))
        E, S, k, Hd = cfg.experts, cfg.shared_experts, cfg.top_k, cfg.hidden
        x_all = H.make_tokens(cfg, sum(Ts), seed=seed, threads=1)
        t0 = sum(Ts[:rank])
        x = x_all[t0:t0 + Ts[rank]]
        T = x.shape[0]
        L = O.port()
        if T:
            ids, sc, off, gt, gs = O.route(L, x, hl.router_w, hl.router_bias, k, cfg.softmax, cfg.renormalize)
        else:
            off, gt, gs = np.zeros(E + 1, np.int32), np.zeros(0, np.uint32), np.zeros(0, np.float32)
        counts = torch.from_numpy(np.diff(off).astype(np.int32)[expert_of_slot].copy())
        gathered = [torch.empty_like(counts) for _ in range(P)]
        dist.all_gather(gathered, counts)
        counts_all = np.stack([g.numpy() for g in gathered])
        max_tokens = max(Ts)
        plan = H.ep_plan(counts_all, k, rank, max_tokens)
        assert plan.tokens[rank] == T

        # dispatch: routed rows grouped by slot, tokens ascending inside a group
        order = (np.concatenate([np.arange(off[e], off[e + 1]) for e in expert_of_slot]).astype(np.int64)
                 if T else np.zeros(0, np.int64))
        gt, gs = gt[order], gs[order]
        row_expert = np.concatenate([np.full(off[e + 1] - off[e], e) for e in expert_of_slot]) if T else order
        xrows = x[gt.astype(np.int64)] if T else np.zeros((0, Hd), np.float32)
        wrows = gs.astype(np.float32)
        xin = np.zeros((plan.recv_total, Hd), np.float32)
        win = np.zeros(plan.recv_total, np.float32)

        def exchange(send_parts, recv_parts):
            reqs = []
            for peer in range(P):
                sb, rb = send_parts[peer], recv_parts[peer]
                if peer == rank:
                    if rb is not None:
                        rb[...] = sb
                    continue
                if sb is not None and sb.size:
                    reqs.append(dist.isend(torch.from_numpy(np.ascontiguousarray(sb)), peer))
                if rb is not None and rb.size:
                    reqs.append((dist.irecv(torch.from_numpy(rb), peer), rb))
            for r in reqs:
                (r[0] if isinstance(r, tuple) else r).wait()

        so, sr = plan.send_offset, plan.send_rows
        ro, rr = plan.recv_offset, plan.recv_rows
        exchange([xrows[so[p]:so[p] + sr[p]] for p in range(P)], [xin[ro[p]:ro[p] + rr[p]] for p in range(P)])
        exchange([wrows[so[p]:so[p] + sr[p]] for p in range(P)], [win[ro[p]:ro[p] + rr[p]] for p in range(P)])

        # owner: local experts over (source, expert) segments
        yin = np.zeros_like(xin)
        row = 0
        for s in range(P):
            for el in range(plan.local_experts):
                n = int(counts_all[s, plan.first_expert + el])
                if n:
                    y = O.expert_mlp(L, xin[row:row + n], *_expert(local, el))
                    yin[row:row + n] = win[row:row + n, None] * y
                row += n
        assert row == plan.recv_total

        # return to the source rows
        yrows = np.zeros_like(xrows)
        exchange([yin[ro[p]:ro[p] + rr[p]] for p in range(P)], [yrows[so[p]:so[p] + sr[p]] for p in range(P)])

        # combine: ascending expert id per token, then shared experts
        out = np.zeros((T, Hd), np.float32)
        for r in np.lexsort((np.arange(len(gt)), row_expert)) if T else []:
            out[gt[r]] += yrows[r]
        for s in range(S):
            if T:
                out += np.float32(1.0) * O.expert_mlp(L, x, *_expert(local, plan.local_experts + s))
        ref = O.moe_layer_port(hl, x_all)[0][t0:t0 + T]
        q.put((rank, bool(np.array_equal(out, ref)), float(np.abs(out - ref).max()) if T else 0.0))
    except Exception as exc:  # reported to the parent
        q.put((rank, False, repr(exc)))
    finally:
        dist.destroy_process_group()


def _peer_rank_main(rank, P, port, cfg_args, Ts, seed, q, placement=None):
    """The peer-memory layout of hmoe_ep_moe_forward with a registered
    workspace (ep.cu: ep_exchange_kernel, ep_permute_kernel,
    ep_combine_kernel), restated on gloo ranks: every rank derives the plan
    from the exchanged counts; each routed row is stored by its source at
    row dest_base[q] + r - send_off[q] of its owner q's receive rows; the
    owner runs its experts over (source, slot) segments in receive order; the
    source reads each output back from the owner at the same row."""
    for p in PATHS:
        sys.path.insert(0, p)
    import torch.distributed as dist

    import hmoe_api as H
    import oracle as O

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=P, timeout=timedelta(seconds=120))
    try:
        cfg = H.LayerConfig(*cfg_args)
        hl = H.make_host_layer(cfg, seed=seed, threads=1)
        local = H.local_host_layer(hl, P, rank, placement)
        expert_of_slot = (np.argsort(np.asarray(placement)) if placement is not None
                          else np.arange(cfg.experts))
        E, S, k, Hd = cfg.experts, cfg.shared_experts, cfg.top_k, cfg.hidden
        x_all = H.make_tokens(cfg, sum(Ts), seed=seed, threads=1)
        t0 = sum(Ts[:rank])
        x = x_all[t0:t0 + Ts[rank]]
        T = x.shape[0]
        L = O.port()
        if T:
            ids, sc, off, gt, gs = O.route(L, x, hl.router_w, hl.router_bias, k, cfg.softmax, cfg.renormalize)
        else:
            off, gt, gs = np.zeros(E + 1, np.int32), np.zeros(0, np.uint32), np.zeros(0, np.float32)
        counts = np.diff(off).astype(np.int64)[expert_of_slot]  # per slot
        counts_all = np.stack(_all_gather(dist, P, counts))      # [P][E]
        # plan, as ep_exchange_kernel forms it
        base, extra = E // P, E % P
        first = [r * base + min(r, extra) for r in range(P)]
        nslot = [base + (1 if r < extra else 0) for r in range(P)]
        R = np.array([[counts_all[p, first[qq]:first[qq] + nslot[qq]].sum() for qq in range(P)] for p in range(P)])
        send_off = [int(R[rank, :qq].sum()) for qq in range(P)]
        dest_base = [int(R[:rank, qq].sum()) for qq in range(P)]
        recv_base = [int(R[:p, rank].sum()) for p in range(P)]
        recv_total = int(R[:, rank].sum())
        # routed rows in slot order, tokens ascending inside a slot
        order = (np.concatenate([np.arange(off[e], off[e + 1]) for e in expert_of_slot]).astype(np.int64)
                 if T else np.zeros(0, np.int64))
        gt, gs = gt[order], gs[order]
        row_expert = np.concatenate([np.full(off[e + 1] - off[e], e) for e in expert_of_slot]) if T else order

        def owner(r):
            qq = 0
            while qq + 1 < P and r >= send_off[qq] + R[rank, qq]:
                qq += 1
            return qq

        # dispatch: (owner, receive row, x row, weight) -- the stores of ep_permute_kernel
        sent = [(owner(r), dest_base[owner(r)] + r - send_off[owner(r)], int(gt[r]), float(gs[r]))
                for r in range(len(gt))]
        everything = _all_gather_obj(dist, P, (t0, sent))
        xin = np.full((recv_total, Hd), np.nan, np.float32)
        win = np.full(recv_total, np.nan, np.float32)
        for p, (tp, items) in enumerate(everything):
            for (qq, d, tok, wgt) in items:
                if qq != rank:
                    continue
                assert recv_base[p] <= d < recv_base[p] + int(R[p, rank]), (p, d)
                assert np.isnan(win[d])  # each receive row written once
                xin[d] = x_all[tp + tok]
                win[d] = wgt
        assert not np.isnan(win).any()
        # owner: (source, local slot) segments in receive order
        yin = np.zeros_like(xin)
        row = 0
        for p in range(P):
            for el in range(nslot[rank]):
                n = int(counts_all[p, first[rank] + el])
                if n:
                    y = O.expert_mlp(L, xin[row:row + n], *_expert(local, el))
                    yin[row:row + n] = win[row:row + n, None] * y
                row += n
        assert row == recv_total
        # combine: each routed row read back from its owner -- the loads of ep_combine_kernel
        yins = _all_gather_obj(dist, P, yin)
        out = np.zeros((T, Hd), np.float32)
        for r in np.lexsort((np.arange(len(gt)), row_expert)) if T else []:
            qq = owner(int(r))
            out[gt[r]] += yins[qq][dest_base[qq] + int(r) - send_off[qq]]
        for sx in range(S):
            if T:
                out += np.float32(1.0) * O.expert_mlp(L, x, *_expert(local, nslot[rank] + sx))
        ref = O.moe_layer_port(hl, x_all)[0][t0:t0 + T]
        q.put((rank, bool(np.array_equal(out, ref)), float(np.abs(out - ref).max()) if T else 0.0))
    except Exception as exc:  # reported to the parent
        q.put((rank, False, repr(exc)))
    finally:
        dist.destroy_process_group()


def _all_gather(dist, P, arr):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(arr))
    out = [torch.empty_like(t) for _ in range(P)]
    dist.all_gather(out, t)
    return [o.numpy() for o in out]


def _all_gather_obj(dist, P, obj):
    out = [None] * P
    dist.all_gather_object(out, obj)
    return out


def _run(P, cfg_args, Ts, seed=0, placement=None, target=None):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    target = target or _rank_main
    procs = [ctx.Process(target=target, args=(r, P, port, cfg_args, Ts, seed, q, placement)) for r in range(P)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(P):
            rank, ok, info = q.get(timeout=300)
            results[rank] = (ok, info)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for r in range(P):
        assert results[r][0], f"rank {r}: {results[r][1]}"


def test_ep_protocol_c1_two_ranks():
    # C1 layer: H256 E8 k2 I512, softmax + renormalise, ragged token counts
    _run(2, (256, 512, 8, 2, True, True, 0, None), (5, 3))


def test_ep_protocol_shared_uneven_three_ranks():
    # 7 experts on 3 ranks (3, 2, 2), 2 shared experts, Zipf-biased router,
    # no renormalisation, and a rank with no tokens
    _run(3, (128, 128, 7, 2, True, False, 2, 1.1), (4, 0, 3), seed=1)


def test_ep_protocol_with_placement_two_ranks():
    # a scrambled expert placement: rows travel in slot order, the combine
    # still adds each token's rows in ascending expert id
    placement = np.random.default_rng(7).permutation(8).astype(np.int32)
    _run(2, (256, 512, 8, 2, True, True, 0, None), (6, 4), seed=2, placement=placement)


def test_ep_peer_layout_two_ranks_with_placement():
    # the peer-memory path's row layout on 2 ranks, scrambled placement
    placement = np.random.default_rng(7).permutation(8).astype(np.int32)
    _run(2, (256, 512, 8, 2, True, True, 0, None), (6, 4), seed=2, placement=placement, target=_peer_rank_main)


def test_ep_peer_layout_three_ranks_shared_uneven():
    # 7 experts on 3 ranks (3, 2, 2), 2 shared experts, Zipf-biased router,
    # no renormalisation, and a rank with no tokens
    _run(3, (128, 128, 7, 2, True, False, 2, 1.1), (4, 0, 3), seed=1, target=_peer_rank_main)


def test_balanced_placement():
    for p in PATHS:
        sys.path.insert(0, p)
    import hmoe_api as H
    load = np.array([10.0, 1, 1, 1, 5, 5, 1, 1], np.float64)
    pl = H.ep_balanced_placement(load, 2)
    assert sorted(pl.tolist()) == list(range(8))
    per = [load[(pl >= 4 * r) & (pl < 4 * r + 4)].sum() for r in range(2)]
    assert per == [13.0, 12.0]  # 10+1+1+1 | 5+5+1+1
    # uneven split (60 experts on 8 ranks: 8,8,8,8,7,7,7,7): every slot used once
    pl = H.ep_balanced_placement(np.linspace(1, 2, 60), 8)
    assert sorted(pl.tolist()) == list(range(60))


def test_ep_plan_rejections():
    for p in PATHS:
        sys.path.insert(0, p)
    import hmoe_api as H
    counts = np.array([[1, 1, 2], [0, 3, 1]], np.int32)
    plan = H.ep_plan(counts, 2, 0, 2)
    assert (plan.first_expert, plan.local_experts) == (0, 2)
    assert list(plan.tokens[:2]) == [2, 2]
    assert list(plan.send_rows[:2]) == [2, 2] and list(plan.send_offset[:2]) == [0, 2]
    assert list(plan.recv_rows[:2]) == [2, 3] and list(plan.recv_offset[:2]) == [0, 2]
    assert plan.recv_total == 5
    with pytest.raises(H.HmoeError) as e:
        H.ep_plan(counts, 2, 0, 1)  # a rank with more tokens than max_tokens
    assert e.value.code == 6
    with pytest.raises(H.HmoeError) as e:
        H.ep_plan(np.array([[1, 1, 1], [0, 0, 0]], np.int32), 2, 1, 4)  # 3 rows is not a multiple of k
    assert e.value.code == 1
    with pytest.raises(H.HmoeError):
        H.ep_plan(np.array([[-1, 1, 2], [0, 0, 0]], np.int32), 2, 0, 4)
    assert [H.ep_expert_range(60, 8, r) for r in range(8)] == [
        (0, 8), (8, 8), (16, 8), (24, 8), (32, 7), (39, 7), (46, 7), (53, 7)]


@pytest.mark.parametrize("P", [2, 3, 4, 5, 8])
@pytest.mark.parametrize("E", [7, 60, 128])
def test_ep_peer_plan_matches_layout(P, E):
    """The device transfer plan (ep_exchange_kernel's code, exported as
    hmoe_ep_peer_plan) against the layout the *_peer_* tests restate:
    send ranges in owner order, receive ranges source-major, rows returned
    to the same positions; ragged counts, empty ranks and sources."""
    if E < P:
        pytest.skip("fewer experts than ranks")
    rng = np.random.default_rng(P * 1000 + E)
    counts = rng.integers(0, 40, size=(P, E)).astype(np.int32)
    counts[rng.random((P, E)) < 0.3] = 0
    counts[P - 1] = 0  # a rank with no tokens
    base, extra = E // P, E % P
    first = [r * base + min(r, extra) for r in range(P)]
    nslot = [base + (1 if r < extra else 0) for r in range(P)]
    R = np.array([[counts[p, first[q]:first[q] + nslot[q]].sum() for q in range(P)] for p in range(P)])
    for me in range(P):
        st, plan = H.ep_peer_plan(counts, me, capacity_rows=10 ** 9)
        assert st == 0
        np.testing.assert_array_equal(plan.send_off[:P], [R[me, :q].sum() for q in range(P)])
        np.testing.assert_array_equal(plan.send_rows[:P], R[me, :])
        np.testing.assert_array_equal(plan.dest_base[:P], [R[:me, q].sum() for q in range(P)])
        np.testing.assert_array_equal(plan.recv_base[:P], [R[:p, me].sum() for p in range(P)])
        np.testing.assert_array_equal(plan.recv_rows[:P], R[:, me])
        np.testing.assert_array_equal(plan.ret_off[:P], [R[p, :me].sum() for p in range(P)])
        assert plan.recv_total == R[:, me].sum() and plan.sent_total == R[me].sum()
        # what a source sends to owner q arrives exactly where q expects it from that source
        for q in range(P):
            _, pq = H.ep_peer_plan(counts, q, capacity_rows=10 ** 9)
            assert plan.dest_base[q] == pq.recv_base[me] and plan.send_rows[q] == pq.recv_rows[me]
    # more rows than the receive capacity: rejected on every rank, nothing moves
    cap = int(R.sum(axis=0).max()) - 1
    for me in range(P):
        st, plan = H.ep_peer_plan(counts, me, capacity_rows=cap)
        assert st == 1 and plan.recv_total == 0 and plan.sent_total == 0 and not any(plan.send_rows[:P])
