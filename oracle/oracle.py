"""ctypes access to the two CPU checkers (TEST INFRASTRUCTURE ONLY).

  port()  -> oracle/_build/libhmoe_oracle.so, the C restatement
             (oracle/hmoe_oracle.c) of the reference CPU hot path;
  ref()   -> oracle/_ref/libhmoe_ref.so, the reference's own CPU classes
             compiled from its sources (oracle/Makefile, oracle/ref_harness.cpp).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use
this module; the product path never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PORT_PATH = os.path.join(HERE, "_build", "libhmoe_oracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libhmoe_ref.so")
# the seeded input generator built apart from libhmoe.so (oracle/Makefile)
SYNTH_PATH = os.path.join(HERE, "_build", "libhmoe_synth.so")
# the reference's own CUDA path, timed as the bar to beat (ref_cuda_bench.cpp)
REF_CUDA_BENCH = os.path.join(HERE, "_ref", "ref_cuda_bench")

_port = None
_ref = None

vp, sz, i32, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_float


def reference_dir():
    """The reference's source tree: $HMOE_REFERENCE, else a checkout named
    `reference` beside this repository; None when neither holds `src/`
    (e.g. on a GPU box, which uses the prebuilt oracle/_ref)."""
    d = os.environ.get("HMOE_REFERENCE") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return d if os.path.isdir(os.path.join(d, "src")) else None


def build(reference: bool = True) -> None:
    """Builds the port (always) and the reference library (when its sources exist)."""
    targets = ["oracle"]
    env = dict(os.environ)
    ref_dir = reference_dir()
    if reference and ref_dir:
        targets.append("ref")
        env["REF"] = ref_dir
    subprocess.run(["make", "-C", HERE, "-j8", *targets], check=True, env=env,
                   stdout=subprocess.DEVNULL)


def _p(a):
    return 0 if a is None else a.ctypes.data


def port() -> ctypes.CDLL:
    global _port
    if _port is None:
        if not os.path.exists(PORT_PATH):
            build(reference=False)
        L = ctypes.CDLL(PORT_PATH)
        L.hmo_route_batch.argtypes = [vp, vp, vp, sz, sz, sz, sz, ctypes.c_int, ctypes.c_int,
                                      vp, vp, vp, vp, vp, vp]
        L.hmo_int8_matmul.argtypes = [vp, vp, vp, sz, sz, sz, f32, i32]
        L.hmo_int8_matmul.restype = None
        L.hmo_expert_mlp.argtypes = [vp, sz, sz, sz, vp, vp, vp, vp, vp, vp]
        L.hmo_expert_mlp.restype = None
        L.hmo_moe_layer.argtypes = [vp, sz, sz, sz, sz, sz, ctypes.c_int, ctypes.c_int, vp, vp, sz,
                                    vp, sz, sz, sz, sz, vp, vp, vp, vp, vp, vp]
        L.hmo_moe_layer_threads.argtypes = L.hmo_moe_layer.argtypes + [ctypes.c_int]
        L.hmo_quantize_int8.argtypes = [vp, sz, vp, vp, vp, vp]
        L.hmo_silu.argtypes = [f32]
        L.hmo_silu.restype = f32
        L.hmo_rms_norm.argtypes = [vp, vp, vp, sz, sz, f32]
        L.hmo_expf_array.argtypes = [vp, vp, sz]
        L.hmo_expf_array.restype = None
        L.hmo_rms_norm.restype = None
        _port = L
    return _port


def ref() -> ctypes.CDLL:
    global _ref
    if _ref is None:
        if not os.path.exists(REF_PATH):
            raise FileNotFoundError(f"{REF_PATH} is not built (needs the reference sources)")
        L = ctypes.CDLL(REF_PATH)
        L.hmr_route_batch.argtypes = [vp, vp, vp, sz, sz, sz, sz, ctypes.c_int, ctypes.c_int,
                                      vp, vp, vp, vp, vp]
        L.hmr_int8_matmul.argtypes = [vp, vp, vp, sz, sz, sz, f32, i32]
        L.hmr_expert_mlp.argtypes = [vp, sz, sz, sz, vp, vp, vp, vp, vp, vp]
        L.hmr_quantize_int8.argtypes = [vp, sz, vp, vp, vp, vp]
        L.hmr_rms_norm.argtypes = [vp, vp, vp, sz, sz, f32]
        L.hmr_layer_create.argtypes = [sz, sz, sz, sz, ctypes.c_int, ctypes.c_int, vp, vp, sz, vp, sz,
                                       sz, sz, sz, vp, vp]
        L.hmr_layer_create.restype = vp
        L.hmr_layer_destroy.argtypes = [vp]
        L.hmr_layer_destroy.restype = None
        L.hmr_layer_forward.argtypes = [vp, vp, sz, vp, vp, vp, vp, ctypes.c_int]
        _ref = L
    return _ref


def ref_available() -> bool:
    return os.path.exists(REF_PATH)


class OracleError(RuntimeError):
    pass


# ------------------------------------------------------------- wrappers

def route(lib, x, w, bias, k, softmax=True, renorm=True):
    """(ids [T,k] u32, scores [T,k] f32, offsets [E+1], group_tokens, group_scores)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    T, H = x.shape
    E = w.shape[1]
    ids = np.zeros((T, k), np.uint32)
    sc = np.zeros((T, k), np.float32)
    off = np.zeros(E + 1, np.int32)
    gt = np.zeros(T * k, np.uint32)
    gs = np.zeros(T * k, np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, np.float32)
    if lib is port():
        st = lib.hmo_route_batch(_p(x), _p(w), _p(b), T, H, E, k, int(softmax), int(renorm),
                                 _p(ids), _p(sc), _p(off), _p(gt), _p(gs), None)
    else:
        st = lib.hmr_route_batch(_p(x), _p(w), _p(b), T, H, E, k, int(softmax), int(renorm),
                                 _p(ids), _p(sc), _p(off), _p(gt), _p(gs))
    if st != 0:
        raise OracleError(f"route failed with status {st}")
    return ids, sc, off, gt, gs


def int8_matmul(lib, left, q, scale, zp):
    left = np.ascontiguousarray(left, np.float32)
    q = np.ascontiguousarray(q, np.int8)
    rows, K = left.shape
    N = q.shape[1]
    out = np.zeros((rows, N), np.float32)
    if lib is port():
        lib.hmo_int8_matmul(_p(left), _p(q), _p(out), rows, K, N, scale, zp)
    else:
        st = lib.hmr_int8_matmul(_p(left), _p(q), _p(out), rows, K, N, scale, zp)
        if st != 0:
            raise OracleError(f"int8 matmul failed with status {st}")
    return out


def expert_mlp(lib, x, gate, up, down, scales, zps):
    x = np.ascontiguousarray(x, np.float32)
    rows, H = x.shape
    I = gate.shape[1]
    y = np.zeros((rows, H), np.float32)
    s = np.ascontiguousarray(scales, np.float32)
    z = np.ascontiguousarray(zps, np.int32)
    args = (_p(x), rows, H, I, _p(np.ascontiguousarray(gate)), _p(np.ascontiguousarray(up)),
            _p(np.ascontiguousarray(down)), _p(s), _p(z), _p(y))
    if lib is port():
        lib.hmo_expert_mlp(*args)
    else:
        st = lib.hmr_expert_mlp(*args)
        if st != 0:
            raise OracleError(f"expert mlp failed with status {st}")
    return y


def quantize(lib, w):
    w = np.ascontiguousarray(w, np.float32)
    q = np.zeros(w.shape, np.int8)
    s, z, e = ctypes.c_float(), ctypes.c_int32(), ctypes.c_float()
    fn = lib.hmo_quantize_int8 if lib is port() else lib.hmr_quantize_int8
    st = fn(_p(w), w.size, _p(q), ctypes.byref(s), ctypes.byref(z), ctypes.byref(e))
    if st != 0:
        raise OracleError(f"quantize failed with status {st}")
    return q, s.value, z.value, e.value


def moe_layer_port(host_layer, x, threads=None):
    """Full layer through the C port: (out [T,H], ids, scores, offsets).
    Expert MLPs run on `threads` host threads (default: every core); the
    result is bit-identical for any thread count."""
    L = port()
    c = host_layer.cfg
    x = np.ascontiguousarray(x, np.float32)
    T = x.shape[0]
    out = np.zeros((T, c.hidden), np.float32)
    ids = np.zeros((T, c.top_k), np.uint32)
    sc = np.zeros((T, c.top_k), np.float32)
    off = np.zeros(c.experts + 1, np.int32)
    st = L.hmo_moe_layer_threads(_p(x), T, c.hidden, c.intermediate, c.experts, c.top_k, int(c.softmax),
                                 int(c.renormalize), _p(host_layer.router_w), _p(host_layer.router_bias),
                                 c.shared_experts, _p(host_layer.arena), c.expert_stride, 0, c.proj_bytes,
                                 2 * c.proj_bytes, _p(host_layer.scales), _p(host_layer.zps), _p(out), _p(ids),
                                 _p(sc), _p(off), int(threads or os.cpu_count() or 1))
    if st != 0:
        raise OracleError(f"moe layer failed with status {st}")
    return out, ids, sc, off


def expf_host(x):
    """The host libm's expf of every element (float32 in, float32 out)."""
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    port().hmo_expf_array(_p(x), _p(out), x.size)
    return out


def rms_norm_port(x, w, eps):
    """RMSNorm through the C port (RMSNorm.cpp:64-77): [T, H] FP32."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    port().hmo_rms_norm(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], float(eps))
    return out


def rms_norm_ref(x, w, eps):
    """RMSNorm through the reference's own RMSNorm class on its CPU backend."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out = np.empty_like(x)
    st = ref().hmr_rms_norm(_p(x), _p(w), _p(out), x.shape[0], x.shape[1], float(eps))
    if st != 0:
        raise OracleError(f"hmr_rms_norm failed with status {st}")
    return out


class RefLayer:
    """A resident layer inside the reference's own CPU classes."""

    def __init__(self, host_layer):
        c = host_layer.cfg
        self.cfg = c
        self._keep = host_layer
        self.handle = ref().hmr_layer_create(
            c.hidden, c.intermediate, c.experts, c.top_k, int(c.softmax), int(c.renormalize),
            _p(host_layer.router_w), _p(host_layer.router_bias), c.shared_experts, _p(host_layer.arena),
            c.expert_stride, 0, c.proj_bytes, 2 * c.proj_bytes, _p(host_layer.scales), _p(host_layer.zps))
        if not self.handle:
            raise OracleError("hmr_layer_create failed")

    def forward(self, x, threads=1, want_routing=False):
        c = self.cfg
        x = np.ascontiguousarray(x, np.float32)
        T = x.shape[0]
        out = np.zeros((T, c.hidden), np.float32)
        ids = np.zeros((T, c.top_k), np.uint32) if want_routing else None
        sc = np.zeros((T, c.top_k), np.float32) if want_routing else None
        off = np.zeros(c.experts + 1, np.int32) if want_routing else None
        st = ref().hmr_layer_forward(self.handle, _p(x), T, _p(out), _p(ids), _p(sc), _p(off), threads)
        if st != 0:
            raise OracleError(f"hmr_layer_forward failed with status {st}")
        return (out, ids, sc, off) if want_routing else out

    def __del__(self):
        if getattr(self, "handle", None):
            ref().hmr_layer_destroy(self.handle)
            self.handle = None
