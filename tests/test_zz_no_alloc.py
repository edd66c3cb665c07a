"""hmoe_moe_forward_noalloc (scratch in a static device array, no caller
workspace) against hmoe_moe_forward on the same inputs: two calls in a row
must both equal the workspace entry point bit for bit, the device status
word it leaves in the static scratch must read back through
hmoe_noalloc_read_status (zero after a clean call, HMOE_NON_FINITE_ROUTER
after a NaN or Inf router input), and a batch beyond the 16 MiB scratch must
be refused.  Collected last so it also runs after every other GPU test in
the same process."""
import ctypes

import numpy as np
import pytest

import hmoe_api as H

pytestmark = pytest.mark.gpu


def noalloc_status():
    import torch
    st, ties, seq = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
    H.check("hmoe_noalloc_read_status", H.lib().hmoe_noalloc_read_status(
        ctypes.byref(st), ctypes.byref(ties), ctypes.byref(seq), torch.cuda.current_stream().cuda_stream))
    return st.value, ties.value, seq.value


@pytest.mark.parametrize("cfg_name,T", [("c1", 64), ("c3", 16), ("c3", 1), ("c2", 3)])
def test_noalloc_forward_matches_workspace_forward(cuda, cfg_name, T):
    import torch
    cfg = H.CONFIGS[cfg_name]
    hl = H.make_host_layer(cfg, seed=11)
    x = torch.from_numpy(H.make_tokens(cfg, T, seed=11)).to(cuda)
    dl = H.DeviceLayer(hl, cuda)
    ref = dl.forward(x).cpu().numpy()
    s = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        y = torch.full((T, cfg.hidden), float("nan"), device=cuda)
        H.check("hmoe_moe_forward_noalloc",
                H.lib().hmoe_moe_forward_noalloc(ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), T, s))
        torch.cuda.synchronize()
        outs.append(y.cpu().numpy())
        assert noalloc_status()[0] == 0
    for y in outs:
        assert np.array_equal(y, ref), float(np.nanmax(np.abs(y - ref)))


@pytest.mark.parametrize("bad", [float("inf"), float("nan")])
def test_noalloc_reports_non_finite_router_input(cuda, bad):
    import torch
    cfg = H.CONFIGS["c1"]
    dl = H.DeviceLayer(H.make_host_layer(cfg, seed=3), cuda)
    x_np = H.make_tokens(cfg, 8, seed=3)
    x_np[5, 17] = bad
    x = torch.from_numpy(x_np).to(cuda)
    y = torch.empty_like(x)
    s = torch.cuda.current_stream().cuda_stream
    H.check("hmoe_moe_forward_noalloc",
            H.lib().hmoe_moe_forward_noalloc(ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), 8, s))
    assert noalloc_status()[0] == 2  # HMOE_NON_FINITE_ROUTER
    assert noalloc_status()[0] == 0  # reading resets the word
    x[5, 17] = 0.0
    H.check("hmoe_moe_forward_noalloc",
            H.lib().hmoe_moe_forward_noalloc(ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), 8, s))
    assert noalloc_status()[0] == 0


def test_noalloc_rejects_oversized_batch(cuda):
    import torch
    cfg = H.CONFIGS["c3"]
    hl = H.make_host_layer(cfg, seed=11)
    dl = H.DeviceLayer(hl, cuda)
    T = 512
    x = torch.zeros((T, cfg.hidden), device=cuda)
    y = torch.zeros((T, cfg.hidden), device=cuda)
    rc = H.lib().hmoe_moe_forward_noalloc(ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), T,
                                          torch.cuda.current_stream().cuda_stream)
    assert rc == 6  # HMOE_WORKSPACE_TOO_SMALL
    assert b"16 MiB" in H.lib().hmoe_last_error()


def test_two_devices_in_one_process():
    """Per-device state (shared-memory limits of every kernel, the static
    no-allocation scratch, the SM count) is kept per device: one process
    runs the tensor-core GEMM path, the single-kernel decode layer and the
    no-allocation entry point on device 0, then on device 1, with the same
    results bit for bit."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = H.CONFIGS["c3"]
    hl = H.make_host_layer(cfg, seed=13)
    results = []
    for ordinal in (0, 1):
        dev = torch.device("cuda", ordinal)
        with torch.cuda.device(dev):
            dl = H.DeviceLayer(hl, dev)
            res = []
            for T in (150, 1, 4):  # GEMM, decode layer, GEMV (all within the 16 MiB scratch)
                x = torch.from_numpy(H.make_tokens(cfg, T, seed=13 + T)).to(dev)
                res.append(dl.forward(x).cpu().numpy())
                y = torch.full((T, cfg.hidden), float("nan"), device=dev)
                H.check("hmoe_moe_forward_noalloc", H.lib().hmoe_moe_forward_noalloc(
                    ctypes.byref(dl.desc), x.data_ptr(), y.data_ptr(), T, torch.cuda.current_stream(dev).cuda_stream))
                torch.cuda.synchronize(dev)
                assert np.array_equal(y.cpu().numpy(), res[-1])
                assert noalloc_status()[0] == 0
                assert dl.read_status()[0] == 0
            results.append(res)
    for a, b in zip(results[0], results[1]):
        assert np.array_equal(a, b)
