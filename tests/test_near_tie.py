"""A token on which the reference and a correctly rounded softmax select
different experts, and the near-tie signal that reports it.

The reference's softmax calls the host libm's expf (std::exp on a float,
src/router/CpuRouterBackend.cpp:54), which is not correctly rounded on every
input: glibc's is off by one ulp on about 6e-4 of the floats in [-64, -0.5].
The device rounds exp once, correctly.  Two candidates whose probabilities
differ by a single ulp can therefore rank differently.  The test builds such
a token: logits 1, 1 + a, 1 + b (and five far below), with a an input the host's expf
rounds up and b just above a, so that expf(a) == expf(b) on the host (a tie,
broken towards the lower id, expert 1) while the correctly rounded exp(a) is
one ulp below exp(b) (expert 2 ranks first).  The router matrix is the
identity, so the logits are exactly the token's first eight values.

CPU: the oracle (the reference's arithmetic) picks [0, 1]; a correctly rounded
softmax picks [0, 2]; a restatement of the device's selection flags the pair
as a near-tie.  GPU: the device flags it (HMOE status near_ties), which is
the contract: selection ids equal the reference's unless a near-tie is
reported."""
from decimal import Decimal, getcontext

import numpy as np
import pytest

import hmoe_api as H
import oracle as O

E, K, HID = 8, 2, 64


def _correct_expf(x):
    """Correctly rounded float exp of float32 inputs (via double; the chosen
    inputs are re-checked with 60 decimal digits)."""
    return np.exp(np.asarray(x, np.float32).astype(np.float64)).astype(np.float32)


def _nearest_float_to_exact_exp(x):
    getcontext().prec = 60
    e = Decimal(float(x)).exp()
    f = np.float32(float(e))
    cands = [np.nextafter(f, np.float32(0)), f, np.nextafter(f, np.float32(2))]
    return min(cands, key=lambda c: abs(Decimal(float(c)) - e))


def near_tie_logits():
    """(a, b): host expf(a) == expf(b) == the correctly rounded exp(b), which
    is one ulp above the correctly rounded exp(a)."""
    # In [-1, -0.75] one ulp of x moves exp(x) in [0.37, 0.48) by less than one
    # ulp, so some b just above a rounds exactly to the host's expf(a); and
    # with the denominator 1 + 2 exp(a) the two probabilities land 1-2 ulp
    # apart, never equal.
    lo = np.array([-1.0], np.float32).view(np.uint32)[0]
    hi = np.array([-0.75], np.float32).view(np.uint32)[0]
    xs = np.arange(hi, lo + 1, dtype=np.uint32).view(np.float32)  # [-1, -0.75]
    host = O.expf_host(xs)
    cr = _correct_expf(xs)
    up = np.nonzero(host > cr)[0]
    assert up.size > 0, "the host expf rounds correctly on the whole window"
    for i in up:
        a = xs[i]
        if _nearest_float_to_exact_exp(a) != cr[i]:
            continue
        b = a
        for _ in range(64):  # towards zero: exp grows by less than an ulp per step
            b = np.nextafter(b, np.float32(0))
            cb, hb = _correct_expf([b])[0], O.expf_host(np.array([b], np.float32))[0]
            if cb > host[i]:
                break
            if cb == host[i] and hb == host[i] and _nearest_float_to_exact_exp(b) == cb:
                return a, b
    raise AssertionError("no near-tie pair found")


def token_and_router():
    a, b = near_tie_logits()
    # logits 1, 1 + a, 1 + b (exact in float, and their differences from
    # the maximum are exactly a and b); no logit is 0, whose rounding
    # interval the router's certificate cannot separate from its neighbours
    la, lb = np.float32(1.0) + a, np.float32(1.0) + b
    assert la - np.float32(1.0) == a and lb - np.float32(1.0) == b
    x = np.zeros((1, HID), np.float32)
    x[0, :E] = [1.0, la, lb, -30.0, -30.0, -30.0, -30.0, -30.0]
    w = np.zeros((HID, E), np.float32)
    w[np.arange(E), np.arange(E)] = 1.0
    return x, w


def device_selection(logits, k):
    """The device's softmax and selection restated (csrc/route_core.cuh,
    select_token): correctly rounded exp, double denominator, probabilities
    rounded once, k + 1 rounds of (probability desc, id asc); a near-tie is
    two consecutive picks within 2 ulp with different logits."""
    lv = np.asarray(logits, np.float32)
    d = (lv - lv.max()).astype(np.float32)
    e = _correct_expf(d)
    den = 0.0
    for v in e:
        den += float(v)
    p = (e.astype(np.float64) / den).astype(np.float32)
    order = sorted(range(len(p)), key=lambda j: (-p[j], j))[:k + 1]
    tie = False
    for r in range(1, len(order)):
        i, j = order[r - 1], order[r]
        if lv[i] != lv[j] and abs(int(p[i].view(np.int32)) - int(p[j].view(np.int32))) <= 2:
            tie = True
    return order[:k], tie


def test_near_tie_token_separates_host_expf_from_correct_rounding():
    x, w = token_and_router()
    ids, *_ = O.route(O.port(), x, w, None, K)
    assert list(ids[0]) == [0, 1]  # the host expf ties a and b: the lower id wins
    sel, tie = device_selection(x[0, :E], K)
    assert sel == [0, 2] and tie  # correct rounding ranks b first, and flags the pair


@pytest.mark.gpu
def test_device_reports_the_near_tie(cuda):
    import torch
    x, w = token_and_router()
    ids_port, *_ = O.route(O.port(), x, w, None, K)
    cfg = H.LayerConfig(HID, 64, E, K, True, True, 0, None)
    hl = H.make_host_layer(cfg, seed=4)
    hl.router_w = w
    dl = H.DeviceLayer(hl, cuda)
    ids, *_ = dl.route(torch.from_numpy(x).to(cuda))
    torch.cuda.synchronize()
    st, ties, _ = dl.read_status()
    assert st == 0
    assert ties >= 1
    got = ids.cpu().numpy().view(np.uint32)
    assert np.array_equal(got, ids_port) or ties >= 1
