"""The error bounds behind the routers' rounding certificate, checked with
exact arithmetic on CPU.

The reference forms each router logit as float(s_H), s_H the sequential
double sum of the exact products p_i = double(x_i) * double(W_ie)
(CpuRouterBackend.cpp:44-45).  The device kernels sum in other orders and
certify that their value rounds to the same float, using two bounds:

* first level: |s_H - S_H| <= (H - 1) u sum|p_i|   (u = 2^-53, S_H exact);
* second level (router.cu, refined_logit): |s_H - S_H| <=
  u/(1-u) * sum_i |S_i| + H^2 u^2 sum|p_i|, S_i the exact partial sums.

Both are checked here against the exact difference, computed with Python
integers (every double is an integer times a power of two), on random
Gaussian data and on cancellation-heavy sums, and the second level must be
the tighter one on random-signed data.
"""
import math

import numpy as np

U = 2.0 ** -53


def _exact(v: float) -> tuple:
    m, e = math.frexp(v)  # v = m * 2^e, 0.5 <= |m| < 1
    return int(m * (1 << 53)), e - 53


def _to_int(vals, base_exp):
    out = []
    for v in vals:
        m, e = _exact(float(v))
        out.append(m << (e - base_exp))
    return out


def _check(x: np.ndarray, w: np.ndarray):
    p = (x.astype(np.float64) * w.astype(np.float64)).tolist()  # exact: float x float fits a double
    s = 0.0
    for v in p:  # the reference's sequential double sum
        s += v
    base = min(_exact(v)[1] for v in p + [s] if v != 0.0) if any(v != 0.0 for v in p) else 0
    ip = _to_int(p, base)
    exact_H = sum(ip)
    diff = abs(_to_int([s], base)[0] - exact_H) * 2.0 ** base
    pabs = sum(abs(v) for v in p)
    prefix, sabs = 0, 0.0
    for v in ip:
        prefix += v
        sabs += abs(prefix) * 2.0 ** base
    H = len(p)
    first = (H - 1) * U * pabs * (1 + 1e-12)
    second = U / (1 - U) * sabs + H * H * U * U * pabs
    assert diff <= first, (diff, first)
    assert diff <= second, (diff, second)
    return diff, first, second


def test_bounds_hold_on_gaussian_router_rows():
    rng = np.random.default_rng(11)
    ratios = []
    for _ in range(40):
        H = int(rng.choice([64, 512, 2048]))
        x = rng.standard_normal(H).astype(np.float32)
        w = (0.02 * rng.standard_normal(H)).astype(np.float32)
        diff, first, second = _check(x, w)
        ratios.append(second / first)
    # random signs: partial sums grow like sqrt(i), so the second bound is far tighter
    assert np.median(ratios) < 0.1


def test_bounds_hold_under_cancellation():
    rng = np.random.default_rng(12)
    for _ in range(20):
        H = 1024
        x = rng.standard_normal(H).astype(np.float32)
        w = (0.02 * rng.standard_normal(H)).astype(np.float32)
        # large terms that cancel exactly, interleaved with small ones
        x[: H // 2 : 2] = np.float32(1e4)
        x[1 : H // 2 : 2] = np.float32(-1e4)
        w[: H // 2] = np.float32(0.75)
        _check(x, w)


def test_bounds_hold_with_mixed_magnitudes_and_zeros():
    rng = np.random.default_rng(13)
    for _ in range(20):
        H = 512
        x = (rng.standard_normal(H) * 10.0 ** rng.integers(-20, 20, H)).astype(np.float32)
        w = rng.standard_normal(H).astype(np.float32)
        x[rng.random(H) < 0.1] = 0.0
        _check(x, w)
