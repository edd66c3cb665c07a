"""ctypes binding of include/hmoe.h (lib/libhmoe.so) plus layer helpers.

Host glue for tests and the benchmark: PyTorch provides device memory and
streams; every computation happens inside libhmoe.so.  Loading fails loudly
when the library has not been built -- there is no fallback path.

The layer helper mirrors how the reference's runtime holds an all-resident
MoE layer: one INT8 expert arena in the ExpertPacker layout
(tools/model_convert/ExpertPacker.cpp:150-247), the router matrix
[H, E] (CpuRouterBackend.cpp:44-45 indexing) and per-projection
QuantizationParameters (Quantization.hpp:19-25).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "lib", "libhmoe.so")

OK = 0
STATUS_NAMES = {
    0: "HMOE_OK", 1: "HMOE_INVALID_ARGUMENT", 2: "HMOE_NON_FINITE_ROUTER",
    3: "HMOE_CUDA_ERROR", 4: "HMOE_NCCL_ERROR", 5: "HMOE_TIMEOUT",
    6: "HMOE_WORKSPACE_TOO_SMALL", 7: "HMOE_UNSUPPORTED",
}

# Every symbol include/hmoe.h declares (checked by tests/test_capi.py).
EXPORTS = [
    "hmoe_last_error", "hmoe_activation", "hmoe_int8_weight_matmul",
    "hmoe_int8_weight_matmul_cooperative", "hmoe_int8_gemm_plan",
    "hmoe_router_topk", "hmoe_gather_rows", "hmoe_scatter_add_rows",
    "hmoe_zero", "hmoe_workspace_size", "hmoe_route", "hmoe_moe_forward",
    "hmoe_set_variant", "hmoe_read_status", "hmoe_synth_normal",
    "hmoe_synth_zipf_bias", "hmoe_quantize_int8", "hmoe_synth_arena",
    "hmoe_set_stage_events", "hmoe_launch_count", "hmoe_moe_forward_host",
    "hmoe_ep_expert_range", "hmoe_ep_plan", "hmoe_ep_unique_id", "hmoe_ep_comm_create",
    "hmoe_ep_comm_destroy", "hmoe_ep_workspace_size", "hmoe_ep_moe_forward", "hmoe_ep_last_plan",
    "hmoe_moe_forward_noalloc", "hmoe_selftest_bounded_wait", "hmoe_ep_set_placement",
    "hmoe_ep_balanced_placement", "hmoe_set_route_variant", "hmoe_ep_register_workspace",
    "hmoe_ep_selftest_flag_wait", "hmoe_ep_read_status", "hmoe_noalloc_read_status",
    "hmoe_moe_forward_residual", "hmoe_ep_peer_plan", "hmoe_ep_moe_forward_residual", "hmoe_rms_norm",
]
EP_MAX_RANKS = 64
EP_UNIQUE_ID_BYTES = 128
HOST_IO = 1 << 62


class HmoeError(RuntimeError):
    def __init__(self, fn: str, code: int, detail: str = ""):
        super().__init__(f"{fn} -> {STATUS_NAMES.get(code, code)} {detail}".strip())
        self.code = code


class ExpertQuant(ctypes.Structure):
    _fields_ = [("scale", ctypes.c_float * 3), ("zero_point", ctypes.c_int32 * 3)]


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("hidden", ctypes.c_uint32), ("intermediate", ctypes.c_uint32),
        ("experts", ctypes.c_uint32), ("top_k", ctypes.c_uint32),
        ("softmax", ctypes.c_int32), ("renormalize", ctypes.c_int32),
        ("shared_experts", ctypes.c_uint32), ("reserved0", ctypes.c_uint32),
        ("router_weight", ctypes.c_void_p), ("router_bias", ctypes.c_void_p),
        ("arena", ctypes.c_void_p), ("expert_stride", ctypes.c_uint64),
        ("gate_offset", ctypes.c_uint64), ("up_offset", ctypes.c_uint64),
        ("down_offset", ctypes.c_uint64), ("quant", ctypes.c_void_p),
        ("ep_rank", ctypes.c_int32), ("ep_size", ctypes.c_int32),
    ]


class EpPlan(ctypes.Structure):
    _fields_ = [
        ("first_expert", ctypes.c_uint32), ("local_experts", ctypes.c_uint32),
        ("tokens", ctypes.c_int64 * EP_MAX_RANKS),
        ("send_rows", ctypes.c_int64 * EP_MAX_RANKS), ("send_offset", ctypes.c_int64 * EP_MAX_RANKS),
        ("recv_rows", ctypes.c_int64 * EP_MAX_RANKS), ("recv_offset", ctypes.c_int64 * EP_MAX_RANKS),
        ("recv_total", ctypes.c_int64),
    ]


class EpPeerPlan(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32 * EP_MAX_RANKS) for n in
                ("send_off", "send_rows", "dest_base", "recv_base", "recv_rows", "ret_off")] + \
               [("recv_total", ctypes.c_int32), ("sent_total", ctypes.c_int32)]


class GemmPlan(ctypes.Structure):
    _fields_ = [("implementation", ctypes.c_int32), ("partitions", ctypes.c_size_t),
                ("blocks", ctypes.c_size_t), ("scratch_elements", ctypes.c_size_t)]


_lib = None


def lib() -> ctypes.CDLL:
    """Loads libhmoe.so (raises if it is missing)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is not built; run `python -c 'import __graft_entry__ as g; g.build()'`")
        L = ctypes.CDLL(LIB_PATH)
        vp, sz, i32, u64, f32 = ctypes.c_void_p, ctypes.c_size_t, ctypes.c_int32, ctypes.c_uint64, ctypes.c_float
        L.hmoe_last_error.restype = ctypes.c_char_p
        sigs = {
            "hmoe_activation": [ctypes.c_int, vp, vp, sz, vp],
            "hmoe_int8_weight_matmul": [vp, vp, vp, sz, sz, sz, f32, i32, vp],
            "hmoe_int8_weight_matmul_cooperative": [vp, vp, vp, vp, sz, sz, sz, sz, f32, i32, vp],
            "hmoe_int8_gemm_plan": [sz, sz, sz, i32, ctypes.POINTER(GemmPlan)],
            "hmoe_router_topk": [vp, sz, sz, sz, ctypes.c_int, ctypes.c_int, vp, vp, vp],
            "hmoe_gather_rows": [vp, vp, vp, sz, sz, vp],
            "hmoe_scatter_add_rows": [vp, vp, vp, vp, sz, sz, vp],
            "hmoe_zero": [vp, sz, vp],
            "hmoe_workspace_size": [ctypes.POINTER(LayerDesc), sz, ctypes.POINTER(sz)],
            "hmoe_route": [ctypes.POINTER(LayerDesc), vp, sz, vp, vp, vp, vp, vp, vp, sz, vp],
            "hmoe_moe_forward": [ctypes.POINTER(LayerDesc), vp, vp, sz, vp, sz, vp],
            "hmoe_moe_forward_host": [ctypes.POINTER(LayerDesc), vp, vp, sz, vp, sz, vp],
            "hmoe_moe_forward_residual": [ctypes.POINTER(LayerDesc), vp, vp, vp, vp, sz, vp, sz, vp],
            "hmoe_set_variant": [i32],
            "hmoe_set_route_variant": [i32],
            "hmoe_read_status": [vp, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32), vp],
            "hmoe_quantize_int8": [vp, sz, vp, vp, vp, vp],
            "hmoe_ep_expert_range": [ctypes.c_uint32, i32, i32, ctypes.POINTER(ctypes.c_uint32),
                                     ctypes.POINTER(ctypes.c_uint32)],
            "hmoe_ep_plan": [vp, ctypes.c_uint32, ctypes.c_uint32, i32, i32, sz, ctypes.POINTER(EpPlan)],
            "hmoe_ep_peer_plan": [vp, ctypes.c_uint32, i32, i32, ctypes.c_int64, ctypes.POINTER(EpPeerPlan)],
            "hmoe_ep_unique_id": [vp, sz],
            "hmoe_ep_comm_create": [vp, i32, i32, i32, ctypes.POINTER(vp)],
            "hmoe_ep_comm_destroy": [vp],
            "hmoe_ep_workspace_size": [ctypes.POINTER(LayerDesc), sz, ctypes.POINTER(sz)],
            "hmoe_ep_moe_forward": [ctypes.POINTER(LayerDesc), vp, vp, vp, sz, sz, vp, sz, vp],
            "hmoe_ep_moe_forward_residual": [ctypes.POINTER(LayerDesc), vp, vp, vp, vp, vp, sz, sz, vp, sz, vp],
            "hmoe_rms_norm": [vp, vp, vp, sz, sz, f32, vp],
            "hmoe_ep_last_plan": [vp, ctypes.POINTER(EpPlan)],
            "hmoe_ep_register_workspace": [vp, vp, sz],
            "hmoe_ep_selftest_flag_wait": [vp, ctypes.c_uint64, ctypes.POINTER(i32)],
            "hmoe_ep_read_status": [vp, ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32), vp],
            "hmoe_moe_forward_noalloc": [ctypes.POINTER(LayerDesc), vp, vp, sz, vp],
            "hmoe_noalloc_read_status": [ctypes.POINTER(i32), ctypes.POINTER(i32), ctypes.POINTER(i32), vp],
            "hmoe_selftest_bounded_wait": [vp, ctypes.c_uint32, vp],
            "hmoe_ep_set_placement": [vp, vp, ctypes.c_uint32],
            "hmoe_ep_balanced_placement": [vp, ctypes.c_uint32, i32, vp],
        }
        for name, args in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int
        L.hmoe_set_stage_events.argtypes = [ctypes.POINTER(ctypes.c_void_p), i32]
        L.hmoe_set_stage_events.restype = ctypes.c_int
        L.hmoe_launch_count.argtypes = []
        L.hmoe_launch_count.restype = ctypes.c_int64
        L.hmoe_synth_normal.argtypes = [u64, u64, f32, vp, sz, ctypes.c_int]
        L.hmoe_synth_normal.restype = None
        L.hmoe_synth_zipf_bias.argtypes = [u64, f32, vp, sz]
        L.hmoe_synth_zipf_bias.restype = None
        L.hmoe_synth_arena.argtypes = [u64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                       ctypes.c_uint32, ctypes.c_uint32, f32, vp, u64, u64, u64, u64,
                                       vp, ctypes.c_int]
        L.hmoe_synth_arena.restype = None
        _lib = L
    return _lib


_synth = None


def use_synth_library(path: str) -> None:
    """Takes the seeded-input functions (synth_normal, synth_zipf_bias,
    make_host_layer, make_tokens) from `path`, a standalone build of the
    same generator source (host/synth.cpp), instead of libhmoe.so.  The
    benchmark's reference arm uses it so that it never loads the product
    library; the values are identical."""
    global _synth
    L = ctypes.CDLL(path)
    u64, f32, vp, sz = ctypes.c_uint64, ctypes.c_float, ctypes.c_void_p, ctypes.c_size_t
    L.hmoe_synth_normal.argtypes = [u64, u64, f32, vp, sz, ctypes.c_int]
    L.hmoe_synth_normal.restype = None
    L.hmoe_synth_zipf_bias.argtypes = [u64, f32, vp, sz]
    L.hmoe_synth_zipf_bias.restype = None
    L.hmoe_synth_arena.argtypes = [u64, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32,
                                   ctypes.c_uint32, ctypes.c_uint32, f32, vp, u64, u64, u64, u64,
                                   vp, ctypes.c_int]
    L.hmoe_synth_arena.restype = None
    _synth = L


def _synth_lib() -> ctypes.CDLL:
    return _synth if _synth is not None else lib()


def check(fn: str, code: int) -> None:
    if code != OK:
        detail = lib().hmoe_last_error().decode(errors="replace") if code == 3 else ""
        raise HmoeError(fn, code, detail)


def _ptr(a) -> int:
    """Data pointer of a numpy array or torch tensor (0 for None)."""
    if a is None:
        return 0
    if isinstance(a, np.ndarray):
        return a.ctypes.data
    return a.data_ptr()


def _stream(stream) -> int:
    if stream is None:
        import torch
        return torch.cuda.current_stream().cuda_stream
    return stream if isinstance(stream, int) else stream.cuda_stream


# ---------------------------------------------------------------- synth

def synth_normal(seed: int, stream: int, sigma: float, shape, threads: int = 0) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    _synth_lib().hmoe_synth_normal(seed, stream, sigma, out.ctypes.data, n, threads or os.cpu_count() or 1)
    return out.reshape(shape)


def synth_zipf_bias(seed: int, alpha: float, E: int) -> np.ndarray:
    out = np.empty(E, dtype=np.float32)
    _synth_lib().hmoe_synth_zipf_bias(seed, alpha, out.ctypes.data, E)
    return out


def quantize_int8(w: np.ndarray):
    w = np.ascontiguousarray(w, dtype=np.float32)
    q = np.empty(w.shape, dtype=np.int8)
    scale = ctypes.c_float()
    zp = ctypes.c_int32()
    err = ctypes.c_float()
    check("hmoe_quantize_int8", lib().hmoe_quantize_int8(
        w.ctypes.data, w.size, q.ctypes.data, ctypes.byref(scale), ctypes.byref(zp), ctypes.byref(err)))
    return q, scale.value, zp.value, err.value


# ---------------------------------------------------------------- layers

@dataclass
class LayerConfig:
    hidden: int
    intermediate: int
    experts: int
    top_k: int
    softmax: bool = True
    renormalize: bool = True
    shared_experts: int = 0
    zipf_alpha: Optional[float] = None  # None: no router bias
    sigma: float = 0.02

    @property
    def proj_bytes(self) -> int:
        return self.hidden * self.intermediate

    @property
    def expert_stride(self) -> int:
        # ExpertPacker: blob = gate|up|down, blob start aligned to 4096.
        return (3 * self.proj_bytes + 4095) // 4096 * 4096


# BASELINE.json configurations (the MoE layer of each).
CONFIGS = {
    "c1": LayerConfig(256, 512, 8, 2, True, True, 0, None),
    "c2": LayerConfig(2048, 1408, 60, 4, True, False, 4, None),
    "c3": LayerConfig(2048, 768, 128, 8, True, True, 0, 1.1),
    "c5": LayerConfig(4096, 1536, 128, 8, True, True, 0, 1.1),
}


@dataclass
class HostLayer:
    """Seeded synthetic layer in host memory (numpy)."""
    cfg: LayerConfig
    router_w: np.ndarray        # [H, E] f32
    router_bias: Optional[np.ndarray]
    arena: np.ndarray           # int8 [(E+S) * stride]
    quant: np.ndarray           # ExpertQuant-compatible structured bytes
    scales: np.ndarray          # [(E+S), 3] f32
    zps: np.ndarray             # [(E+S), 3] i32


def make_host_layer(cfg: LayerConfig, seed: int = 0, layer: int = 0, threads: int = 0) -> HostLayer:
    threads = threads or os.cpu_count() or 1
    H, I, E, S = cfg.hidden, cfg.intermediate, cfg.experts, cfg.shared_experts
    router_w = synth_normal(seed, 2 + (layer << 8), cfg.sigma, (H, E), threads)
    bias = synth_zipf_bias(seed + layer, cfg.zipf_alpha, E) if cfg.zipf_alpha else None
    total = E + S
    stride = cfg.expert_stride
    arena = np.zeros(total * stride, dtype=np.int8)
    quant = (ExpertQuant * total)()
    _synth_lib().hmoe_synth_arena(seed, layer, 0, total, H, I, cfg.sigma, arena.ctypes.data, stride,
                           0, cfg.proj_bytes, 2 * cfg.proj_bytes, ctypes.addressof(quant), threads)
    qbytes = np.frombuffer(bytes(quant), dtype=np.uint8).copy()
    scales = np.array([[quant[e].scale[p] for p in range(3)] for e in range(total)], dtype=np.float32)
    zps = np.array([[quant[e].zero_point[p] for p in range(3)] for e in range(total)], dtype=np.int32)
    return HostLayer(cfg, router_w, bias, arena, qbytes, scales, zps)


def make_tokens(cfg: LayerConfig, T: int, seed: int = 0, threads: int = 0) -> np.ndarray:
    return synth_normal(seed, 1, 1.0, (T, cfg.hidden), threads)


def _check_rows(name, t, T, width, dtype, device=None):
    """The C ABI reads raw pointers: refuse a tensor whose dtype, shape,
    layout or device the kernels would misread (None passes)."""
    if t is None:
        return
    if (t.dtype != dtype or not t.is_contiguous() or t.dim() != 2 or tuple(t.shape) != (T, width)
            or (device is not None and t.device != device)):
        where = f" on {device}" if device is not None else ""
        raise ValueError(f"{name} must be a contiguous {dtype} tensor of shape [{T}, {width}]{where}; "
                         f"got {t.dtype} {tuple(t.shape)} on {t.device}")


class DeviceLayer:
    """A HostLayer resident on the current CUDA device, plus its descriptor."""

    def __init__(self, host: HostLayer, device="cuda"):
        import torch
        cfg = host.cfg
        self.host = host
        self.cfg = cfg
        self.router_w = torch.from_numpy(host.router_w).to(device)
        self.router_bias = torch.from_numpy(host.router_bias).to(device) if host.router_bias is not None else None
        self.arena = torch.from_numpy(host.arena).to(device)
        self.quant = torch.from_numpy(host.quant).to(device)
        d = LayerDesc()
        d.hidden, d.intermediate, d.experts, d.top_k = cfg.hidden, cfg.intermediate, cfg.experts, cfg.top_k
        d.softmax, d.renormalize = int(cfg.softmax), int(cfg.renormalize)
        d.shared_experts = cfg.shared_experts
        d.router_weight = self.router_w.data_ptr()
        d.router_bias = self.router_bias.data_ptr() if self.router_bias is not None else None
        d.arena = self.arena.data_ptr()
        d.expert_stride = cfg.expert_stride
        d.gate_offset, d.up_offset, d.down_offset = 0, cfg.proj_bytes, 2 * cfg.proj_bytes
        d.quant = self.quant.data_ptr()
        d.ep_rank, d.ep_size = 0, 1
        self.desc = d
        self._ws = None

    def _check_io(self, T, x=None, y=None, residual=None, y_bf16=None):
        import torch
        dev, Hd = self.arena.device, self.cfg.hidden
        _check_rows("x", x, T, Hd, torch.float32, dev)
        _check_rows("y", y, T, Hd, torch.float32, dev)
        _check_rows("residual", residual, T, Hd, torch.float32, dev)
        _check_rows("y_bf16", y_bf16, T, Hd, torch.bfloat16, dev)

    def workspace_bytes(self, T: int, host_io: bool = False) -> int:
        n = ctypes.c_size_t()
        check("hmoe_workspace_size", lib().hmoe_workspace_size(
            ctypes.byref(self.desc), T | (HOST_IO if host_io else 0), ctypes.byref(n)))
        return n.value

    def workspace(self, T: int, host_io: bool = False):
        import torch
        need = self.workspace_bytes(T, host_io)
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.empty(need, dtype=torch.uint8, device=self.arena.device)
        return self._ws

    def forward(self, x, y=None, stream=None):
        import torch
        if self.desc.ep_size != 1:
            raise ValueError("expert-parallel layer: use EpLayer.forward")
        T = x.shape[0]
        if y is None:
            y = torch.empty((T, self.cfg.hidden), dtype=torch.float32, device=x.device)
        self._check_io(T, x=x, y=y)
        ws = self.workspace(T)
        check("hmoe_moe_forward", lib().hmoe_moe_forward(
            ctypes.byref(self.desc), x.data_ptr(), y.data_ptr(), T, ws.data_ptr(), ws.numel(), _stream(stream)))
        return y

    def forward_residual(self, x, residual=None, y=None, y_bf16=None, stream=None):
        """y = residual + layer(x) (FP32, one rounding), and optionally its
        BF16 copy y_bf16 (a torch.bfloat16 tensor [T, H])."""
        import torch
        T = x.shape[0]
        if y is None:
            y = torch.empty((T, self.cfg.hidden), dtype=torch.float32, device=x.device)
        self._check_io(T, x=x, y=y, residual=residual, y_bf16=y_bf16)
        ws = self.workspace(T)
        check("hmoe_moe_forward_residual", lib().hmoe_moe_forward_residual(
            ctypes.byref(self.desc), x.data_ptr(), _ptr(residual), y.data_ptr(), _ptr(y_bf16), T,
            ws.data_ptr(), ws.numel(), _stream(stream)))
        return y

    def forward_host(self, x_host, y_host, stream=None, workspace=None):
        """x_host/y_host: page-locked CPU tensors [T, H] FP32.  `workspace`
        (a device uint8 tensor of at least workspace_bytes(T, host_io=True))
        replaces the layer's own, so that calls on different streams can be
        in flight together."""
        import torch
        T = x_host.shape[0]
        for name, t in (("x_host", x_host), ("y_host", y_host)):
            _check_rows(name, t, T, self.cfg.hidden, torch.float32, torch.device("cpu"))
        ws = workspace if workspace is not None else self.workspace(T, host_io=True)
        check("hmoe_moe_forward_host", lib().hmoe_moe_forward_host(
            ctypes.byref(self.desc), x_host.data_ptr(), y_host.data_ptr(), T, ws.data_ptr(), ws.numel(),
            _stream(stream)))
        return y_host

    def route(self, x, stream=None):
        import torch
        T, k, E = x.shape[0], self.cfg.top_k, self.cfg.experts
        self._check_io(T, x=x)
        dev = x.device
        ids = torch.empty((T, k), dtype=torch.int32, device=dev)
        scores = torch.empty((T, k), dtype=torch.float32, device=dev)
        offsets = torch.empty(E + 1, dtype=torch.int32, device=dev)
        gtok = torch.empty(T * k, dtype=torch.int32, device=dev)
        gsc = torch.empty(T * k, dtype=torch.float32, device=dev)
        ws = self.workspace(T)
        check("hmoe_route", lib().hmoe_route(
            ctypes.byref(self.desc), x.data_ptr(), T, ids.data_ptr(), scores.data_ptr(), offsets.data_ptr(),
            gtok.data_ptr(), gsc.data_ptr(), ws.data_ptr(), ws.numel(), _stream(stream)))
        return ids, scores, offsets, gtok, gsc

    def read_status(self, stream=None):
        st, ties, seq = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check("hmoe_read_status", lib().hmoe_read_status(
            self._ws.data_ptr(), ctypes.byref(st), ctypes.byref(ties), ctypes.byref(seq), _stream(stream)))
        return st.value, ties.value, seq.value


def set_variant(v: int) -> None:
    check("hmoe_set_variant", lib().hmoe_set_variant(v))


def set_route_variant(v: int) -> None:
    """0 = automatic, 1 = per-8-token cluster router, 2 = tiled router, 3 = decode router."""
    check("hmoe_set_route_variant", lib().hmoe_set_route_variant(v))


# ------------------------------------------------------ expert parallelism

def ep_expert_range(experts: int, ep_size: int, ep_rank: int):
    """(first, count) of the routed experts rank `ep_rank` owns."""
    f, n = ctypes.c_uint32(), ctypes.c_uint32()
    check("hmoe_ep_expert_range", lib().hmoe_ep_expert_range(experts, ep_size, ep_rank, ctypes.byref(f),
                                                              ctypes.byref(n)))
    return f.value, n.value


def ep_plan(counts: np.ndarray, top_k: int, ep_rank: int, max_tokens: int) -> EpPlan:
    """Transfer plan of `ep_rank` from counts[ep_size, experts] (int32)."""
    counts = np.ascontiguousarray(counts, dtype=np.int32)
    P, E = counts.shape
    plan = EpPlan()
    check("hmoe_ep_plan", lib().hmoe_ep_plan(counts.ctypes.data, E, top_k, P, ep_rank, max_tokens,
                                             ctypes.byref(plan)))
    return plan


def ep_peer_plan(slot_counts: np.ndarray, ep_rank: int, capacity_rows: int):
    """(status, plan) of the peer-memory path's device transfer plan for
    `ep_rank` from slot_counts[ep_size, experts] (int32)."""
    counts = np.ascontiguousarray(slot_counts, dtype=np.int32)
    P, E = counts.shape
    plan = EpPeerPlan()
    st = lib().hmoe_ep_peer_plan(counts.ctypes.data, E, P, ep_rank, capacity_rows, ctypes.byref(plan))
    return st, plan


def ep_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(EP_UNIQUE_ID_BYTES)
    check("hmoe_ep_unique_id", lib().hmoe_ep_unique_id(buf, EP_UNIQUE_ID_BYTES))
    return buf.raw


def ep_balanced_placement(load, ep_size: int) -> np.ndarray:
    """slot_of_expert balancing the expected per-expert `load` over ranks."""
    load = np.ascontiguousarray(load, dtype=np.float64)
    out = np.zeros(load.size, dtype=np.int32)
    check("hmoe_ep_balanced_placement", lib().hmoe_ep_balanced_placement(load.ctypes.data, load.size, ep_size,
                                                                         out.ctypes.data))
    return out


def local_host_layer(host: HostLayer, ep_size: int, ep_rank: int, slot_of_expert=None) -> HostLayer:
    """The slice of `host` that rank `ep_rank` holds: its routed experts (in
    placement-slot order) followed by every shared expert (router replicated)."""
    cfg = host.cfg
    E, S, stride = cfg.experts, cfg.shared_experts, cfg.expert_stride
    f, n = ep_expert_range(E, ep_size, ep_rank)
    if slot_of_expert is None:
        routed = list(range(f, f + n))
    else:
        expert_of_slot = np.argsort(np.asarray(slot_of_expert))
        routed = [int(e) for e in expert_of_slot[f:f + n]]
    ids = routed + list(range(E, E + S))
    arena = np.concatenate([host.arena[e * stride:(e + 1) * stride] for e in ids])
    qsz = ctypes.sizeof(ExpertQuant)
    quant = np.concatenate([host.quant[e * qsz:(e + 1) * qsz] for e in ids])
    return HostLayer(cfg, host.router_w, host.router_bias, arena, quant, host.scales[ids], host.zps[ids])


class EpComm:
    """One rank's NCCL communicator (collective create: every rank calls it
    with the same unique id, on its own device)."""

    def __init__(self, unique_id: bytes, rank: int, size: int, timeout_ms: int = 60000):
        h = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, EP_UNIQUE_ID_BYTES)
        check("hmoe_ep_comm_create", lib().hmoe_ep_comm_create(buf, rank, size, timeout_ms, ctypes.byref(h)))
        self.handle = h
        self.rank, self.size = rank, size

    def set_placement(self, slot_of_expert) -> None:
        if slot_of_expert is None:
            check("hmoe_ep_set_placement", lib().hmoe_ep_set_placement(self.handle, None, 0))
            return
        arr = np.ascontiguousarray(slot_of_expert, dtype=np.int32)
        check("hmoe_ep_set_placement", lib().hmoe_ep_set_placement(self.handle, arr.ctypes.data, arr.size))

    def last_plan(self) -> EpPlan:
        plan = EpPlan()
        check("hmoe_ep_last_plan", lib().hmoe_ep_last_plan(self.handle, ctypes.byref(plan)))
        return plan

    def register_workspace(self, ws) -> None:
        """Collective: peer-memory path for this workspace (None unregisters)."""
        check("hmoe_ep_register_workspace", lib().hmoe_ep_register_workspace(
            self.handle, ws.data_ptr() if ws is not None else None, ws.numel() if ws is not None else 0))

    def selftest_flag_wait(self, limit_ns: int) -> int:
        st = ctypes.c_int32()
        check("hmoe_ep_selftest_flag_wait", lib().hmoe_ep_selftest_flag_wait(self.handle, limit_ns, ctypes.byref(st)))
        return st.value

    def close(self):
        if self.handle:
            h, self.handle = self.handle, None
            check("hmoe_ep_comm_destroy", lib().hmoe_ep_comm_destroy(h))


class EpLayer(DeviceLayer):
    """This rank's share of an expert-parallel layer on the current device."""

    def __init__(self, host: HostLayer, comm: EpComm, device="cuda", slot_of_expert=None, peer: bool = True):
        """peer: register the workspace for the peer-memory path (collective;
        every rank must pass the same value); False keeps the NCCL path."""
        super().__init__(local_host_layer(host, comm.size, comm.rank, slot_of_expert), device)
        comm.set_placement(slot_of_expert)
        self.full_host = host
        self.comm = comm
        self.peer = peer
        self.desc.ep_rank, self.desc.ep_size = comm.rank, comm.size

    def ep_workspace(self, max_tokens: int):
        import torch
        n = ctypes.c_size_t()
        check("hmoe_ep_workspace_size", lib().hmoe_ep_workspace_size(ctypes.byref(self.desc), max_tokens,
                                                                     ctypes.byref(n)))
        if self._ws is None or self._ws.numel() < n.value:
            # every rank sizes the same, so every rank re-registers together
            self._ws = torch.empty(n.value, dtype=torch.uint8, device=self.arena.device)
            if self.peer:
                try:
                    self.comm.register_workspace(self._ws)
                except HmoeError as exc:
                    if exc.code != 7:  # HMOE_UNSUPPORTED: some rank cannot map every peer
                        raise
                    # returned on every rank alike, so every rank keeps the NCCL path
                    import warnings
                    warnings.warn(f"expert parallelism: peer-memory path unavailable ({exc}); using NCCL")
                    self.peer = False
        return self._ws

    def read_status(self, stream=None):
        st, ties, seq = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        check("hmoe_ep_read_status", lib().hmoe_ep_read_status(
            self._ws.data_ptr(), ctypes.byref(st), ctypes.byref(ties), ctypes.byref(seq), _stream(stream)))
        return st.value, ties.value, seq.value

    def forward(self, x, y=None, stream=None, max_tokens: Optional[int] = None):
        import torch
        T = x.shape[0]
        max_tokens = max_tokens or max(T, 1)
        if y is None:
            y = torch.empty((T, self.cfg.hidden), dtype=torch.float32, device=x.device)
        self._check_io(T, x=x, y=y)
        ws = self.ep_workspace(max_tokens)
        check("hmoe_ep_moe_forward", lib().hmoe_ep_moe_forward(
            ctypes.byref(self.desc), self.comm.handle, x.data_ptr() if T else None, y.data_ptr() if T else None,
            T, max_tokens, ws.data_ptr(), ws.numel(), _stream(stream)))
        return y

    def forward_residual(self, x, residual=None, y=None, y_bf16=None, stream=None,
                         max_tokens: Optional[int] = None):
        """Collective: y = residual + layer(x) over the communicator's ranks
        (hmoe_ep_moe_forward_residual); residual and y may alias x."""
        import torch
        T = x.shape[0]
        max_tokens = max_tokens or max(T, 1)
        if y is None:
            y = torch.empty((T, self.cfg.hidden), dtype=torch.float32, device=x.device)
        self._check_io(T, x=x, y=y, residual=residual, y_bf16=y_bf16)
        ws = self.ep_workspace(max_tokens)
        check("hmoe_ep_moe_forward_residual", lib().hmoe_ep_moe_forward_residual(
            ctypes.byref(self.desc), self.comm.handle, x.data_ptr() if T else None,
            _ptr(residual) if T else None, y.data_ptr() if T else None, _ptr(y_bf16) if T else None,
            T, max_tokens, ws.data_ptr(), ws.numel(), _stream(stream)))
        return y


# ------------------------------------------------------------ layer stacks

def make_norm_weight(cfg: LayerConfig, seed: int = 0, layer: int = 0) -> np.ndarray:
    """Seeded RMSNorm weight [H] of layer `layer`'s block: 1 + N(0, 0.1^2)."""
    return (1.0 + synth_normal(seed, (1 << 60) + layer, 0.1, (cfg.hidden,))).astype(np.float32)


def rms_norm(x, weight, out=None, eps: float = 1e-6, stream=None):
    """hmoe_rms_norm over device tensors [T, H] FP32 (out may be x)."""
    import torch
    if out is None:
        out = torch.empty_like(x)
    for name, t in (("x", x), ("weight", weight), ("out", out)):
        if t.dtype != torch.float32 or not t.is_contiguous() or t.device != x.device:
            raise ValueError(f"rms_norm: {name} must be a contiguous FP32 tensor on {x.device}")
    if x.dim() != 2 or out.shape != x.shape or weight.shape != (x.shape[1],):
        raise ValueError("rms_norm: x and out are [T, H], weight is [H]")
    T, Hd = x.shape
    check("hmoe_rms_norm", lib().hmoe_rms_norm(x.data_ptr() if T else None, weight.data_ptr(),
                                               out.data_ptr() if T else None, T, Hd, eps, _stream(stream)))
    return out


class MoEStack:
    """A stack of transformer blocks whose attention is the identity (as in
    MoELayer::execute), i.e. per block the post-attention RMSNorm, the MoE
    layer and its residual add (TransformerBlock::execute,
    src/transformer/runtime/TransformerBlock.cpp:90-104):
        x_{l+1} = x_l + layer_l(rms_norm(x_l) * g_l),  l = 0 .. n_layers-1,
    the add in one FP32 rounding, in place in the caller's buffer.  The norm
    is what keeps a deep stack finite: SwiGLU's output grows with the square
    of its input, so without it the residual stream overflows within a few
    dozen layers.

    Layer l's weights are generated from (seed, l) by make_host_layer and its
    norm weight by make_norm_weight, so the stack is BASELINE's 48-layer
    Qwen3-30B-A3B configuration when built from CONFIGS["c3"] with
    n_layers=48.  Every layer stays resident on the device (no tiering).  All
    layers share one workspace, since they run one after another on one
    stream.  With `comm` the layers are expert-parallel over its ranks
    (EpLayer), sharing the communicator, its expert placement and one
    registered workspace."""

    def __init__(self, cfg: LayerConfig, n_layers: int, seed: int = 0, device="cuda", comm=None,
                 slot_of_expert=None, peer: bool = True, hosts=None, eps: float = 1e-6):
        """hosts: an iterable of the layers' HostLayers (a list the caller
        keeps to compare against, or a generator); by default each layer is
        generated from (seed, layer), uploaded and dropped, so host memory
        holds one layer at a time.  eps: RMSNorm's epsilon (its default,
        src/transformer/norm/RMSNorm.hpp:18)."""
        import torch
        self.cfg = cfg
        self.comm = comm
        self.eps = eps
        self.layers = []
        self.norm_host = [make_norm_weight(cfg, seed, l) for l in range(n_layers)]
        self.norm_w = [torch.from_numpy(g).to(device) for g in self.norm_host]
        it = iter(hosts) if hosts is not None else (make_host_layer(cfg, seed=seed, layer=l)
                                                    for l in range(n_layers))
        for _ in range(n_layers):
            host = next(it)
            if comm is None:
                layer = DeviceLayer(host, device)
            else:
                layer = EpLayer(host, comm, device, slot_of_expert=slot_of_expert, peer=peer)
                layer.full_host = None
            layer.host = None
            self.layers.append(layer)
            del host
        self._ws = None
        self._xn = None

    def _share_workspace(self, T: int, max_tokens: Optional[int]):
        import torch
        first = self.layers[0]
        if self.comm is None:
            need = first.workspace_bytes(T)
            if self._ws is None or self._ws.numel() < need:
                self._ws = torch.empty(need, dtype=torch.uint8, device=first.arena.device)
        else:
            # the first layer sizes and registers it (collective); the others
            # reuse it, so every layer call takes the same transfer path
            self._ws = first.ep_workspace(max_tokens or max(T, 1))
            for layer in self.layers[1:]:
                layer.peer = first.peer
        for layer in self.layers:
            layer._ws = self._ws

    def forward(self, x, stream=None, max_tokens: Optional[int] = None, trace=None):
        """x [T, H] FP32 on the device, updated in place and returned.
        trace: a list that receives, per layer, host copies of the layer's
        residual input and of its normalised input (tests only: it
        synchronises)."""
        import torch
        if x.dtype != torch.float32 or not x.is_contiguous() or x.dim() != 2 or x.shape[1] != self.cfg.hidden:
            raise ValueError(f"MoEStack.forward: x must be a contiguous FP32 [T, {self.cfg.hidden}] tensor")
        T = x.shape[0]
        self._share_workspace(T, max_tokens)
        if self._xn is None or self._xn.shape[0] < T:
            self._xn = torch.empty((max(T, 1), self.cfg.hidden), dtype=torch.float32, device=x.device)
        xn = self._xn[:T]
        for l, layer in enumerate(self.layers):
            rms_norm(x, self.norm_w[l], out=xn, eps=self.eps, stream=stream)
            if trace is not None:
                trace.append((x.cpu().numpy().copy(), xn.cpu().numpy().copy()))
            if self.comm is None:
                layer.forward_residual(xn, residual=x, y=x, stream=stream)
            else:
                layer.forward_residual(xn, residual=x, y=x, stream=stream, max_tokens=max_tokens)
        return x

    def read_status(self, stream=None):
        return self.layers[0].read_status(stream)
