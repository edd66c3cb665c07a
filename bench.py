#!/usr/bin/env python
"""MoE-layer tokens/s on B200: the Qwen3-30B-A3B-shaped layer with INT8 experts.

Workload: hidden 2048, 128 routed experts, top-8 with
renormalised probabilities, expert intermediate 768, SwiGLU, INT8
per-projection affine expert weights quantised from seeded N(0, 0.02^2),
Zipf(1.1)-skewed router logits, activations ~N(0,1), 4096 tokens per GPU per
step (the prefill batch; --tokens picks 1/16/256 for decode-sized batches).
Seeded synthetic inputs stand in for real checkpoints and prompts.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--tokens T]
  python bench.py --impl reference ...    the reference's own CPU path

One JSON line on rank 0.  `value` is device-timed (CUDA events per step,
inputs resident in HBM, L2 flushed between steps); `e2e` is the same metric
through hmoe_moe_forward_host with page-locked host buffers, both copies
inside the timed region, with three calls in flight on three streams (a
batch's copies overlap another batch's layer); `e2e_serial` is one call at
a time.  `roofline` covers the dominant stage, timed live
with events the library records at stage boundaries.  `cpu_baseline` is the
reference's own CPU implementation (oracle/_ref, compiled from its sources)
on a bounded token sample, on this host's cores.

Multi-GPU (torchrun, one process per GPU): expert parallelism through
hmoe_ep_moe_forward.  Rank r holds its contiguous share of the 128 routed
experts and routes its own 4096 tokens (weak scaling); rows travel to the
expert owners and back as stores into the peers' memory over NVLink
(registered workspaces, epoch flags; --ep-path nccl: NCCL point-to-point
instead).  The step time is the max over ranks.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from typing import Optional

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "hypermoe-engine_b200"))

METRIC = "MoE-layer tokens/s (Qwen3-30B-A3B shape, INT8 experts)"
WORKLOADS = {"c1": "c1: small cpu-runnable moe layer", "c2": "c2: qwen1.5-moe-a2.7b moe layer (4 shared experts)",
             "c3": "c3: qwen3-30b-a3b moe layer", "c5": "c5: qwen3-235b-a22b moe layer"}
SHAPES = {"c1": "H256 E8 k2 I512", "c2": "Qwen1.5-MoE-A2.7B shape", "c3": "Qwen3-30B-A3B shape",
          "c5": "Qwen3-235B-A22B shape"}
UNIT = "tokens/s"
STAGES = ["route", "group", "gate_up", "down", "combine"]


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--tokens", type=int, default=None,
                   help="tokens per GPU (default 4096; c4: the 2048-token prefill)")
    p.add_argument("--config", default="c3",
                   help="c1/c2/c3/c5: one MoE layer; c4: the 48-layer Qwen3-30B-A3B stack of c3 layers")
    p.add_argument("--layers", type=int, default=48, help="c4: layers in the stack")
    p.add_argument("--decode-batch", type=int, default=64, help="c4: decode batch over all GPUs")
    p.add_argument("--stack-cpu-tokens", type=int, default=8,
                   help="c4: tokens the reference CPU path runs through the whole stack")
    p.add_argument("--no-stack", action="store_true",
                   help="single GPU: skip the c4 stack and the c2/c5 layer measurements added to the c3 line")
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--impl", default="hmoe", choices=["hmoe", "reference"])
    p.add_argument("--variant", type=int, default=0,
                   help="0 auto, 1 GEMV only, 2 GEMM only, 3 single-kernel decode layer (T <= 8)")
    p.add_argument("--route-variant", type=int, default=0, help="0 auto, 1 cluster router, 2 tiled router")
    p.add_argument("--ep-path", default="peer", choices=["peer", "nccl"],
                   help="expert parallelism: peer-memory stores (registered workspace) or NCCL send/recv")
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-reference-cuda", action="store_true",
                   help="skip timing the reference's own CUDA path on this GPU")
    p.add_argument("--cpu-seconds", type=float, default=12.0)
    p.add_argument("--placement", default="balanced", choices=["balanced", "contiguous"],
                   help="expert placement under expert parallelism: balanced from a calibration batch's "
                        "routing counts (EPLB-style static placement), or contiguous expert ids")
    p.add_argument("--no-e2e", action="store_true",
                   help="skip the host-buffer (e2e) measurements (e.g. for a kernel launch list)")
    p.add_argument("--no-decode", action="store_true",
                   help="skip the decode-size stage splits added to a prefill line")
    p.add_argument("--decode-tokens", default="1,8,16",
                   help="comma-separated decode batch sizes for the stage splits of a prefill line")
    p.add_argument("--eager", action="store_true",
                   help="time eager hmoe_moe_forward calls instead of CUDA-graph replays")
    return p.parse_args()


def metric_for(config: str) -> str:
    """BASELINE's metric for the c3 workload; the same wording for the others."""
    return METRIC if config == "c3" else f"MoE-layer tokens/s ({SHAPES.get(config, config)}, INT8 experts)"


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """SM clock and throttle-reason sampler for the timed region (read-only
    NVML queries every 5 ms; nvidia-smi every 200 ms when NVML is missing)."""

    REASONS = {"hw_slowdown": "nvmlClocksEventReasonHwSlowdown",
               "hw_thermal_slowdown": "nvmlClocksEventReasonHwThermalSlowdown",
               "sw_thermal_slowdown": "nvmlClocksEventReasonSwThermalSlowdown",
               "sw_power_cap": "nvmlClocksEventReasonSwPowerCap"}
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int, pci_bus_id: Optional[str] = None):
        self.index = index
        self.pci = pci_bus_id
        self.proc = None
        self.thread = None
        self.stop_flag = threading.Event()
        self.sm, self.max_mhz, self.reasons = [], None, set()
        self.lines = []

    def start(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            h = (pynvml.nvmlDeviceGetHandleByPciBusId(self.pci.encode()) if self.pci
                 else pynvml.nvmlDeviceGetHandleByIndex(self.index))
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
            bits = {n: getattr(pynvml, v) for n, v in self.REASONS.items()}

            def poll():
                while not self.stop_flag.is_set():
                    self.sm.append(float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)))
                    r = pynvml.nvmlDeviceGetCurrentClocksEventReasons(h)
                    for n, bit in bits.items():
                        if r & bit:
                            self.reasons.add(n)
                    time.sleep(0.005)
            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        except Exception:
            pass
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.index)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None and self.thread is not None:  # NVML sampler
            self.stop_flag.set()
            self.thread.join(timeout=2)
            return {"sm_mhz": statistics.median(self.sm) if self.sm else None, "sm_max_mhz": self.max_mhz,
                    "reasons": sorted(self.reasons), "samples": len(self.sm), "source": "nvml 5 ms"}
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["clock sampling unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm), "source": "nvidia-smi 200 ms"}


def algorithmic(cfg, T, U, rows_in=None, local_experts=None):
    """Algorithmic bytes and FLOPs per stage of one layer call on one GPU.

    U: experts with at least one row on this GPU (weights streamed once);
    rows_in: expert rows this GPU computes (T*(k+S) on one GPU; the received
    rows plus the shared-expert rows under expert parallelism)."""
    H, I, E, k, S = cfg.hidden, cfg.intermediate, cfg.experts, cfg.top_k, cfg.shared_experts
    rows = T * (k + S)
    rin = rows if rows_in is None else rows_in
    return {
        "route": {"bytes": T * H * 4 + H * E * 4 + T * k * 8, "flops": 2 * T * H * E},
        # grouping ids/scores, then each token row read once and written as
        # FP16 rows (plus a 4-byte scale per row)
        "group": {"bytes": T * k * 8 * 2 + T * H * 4 + rows * (H * 2 + 4), "flops": 0},
        "gate_up": {"bytes": U * 2 * H * I + rin * H * 2 + rin * I * 2, "flops": 4 * rin * H * I},
        "down": {"bytes": U * H * I + rin * I * 2 + rin * H * 2, "flops": 2 * rin * H * I},
        "combine": {"bytes": rows * H * 2 + T * H * 4, "flops": 0},
        "layer": {"bytes": U * 3 * H * I + H * E * 4 + 8 * T * H,
                  "flops": 2 * T * H * E + rin * 6 * H * I},
        "unique_experts": U,
    }


def cpu_reference_sample(cfg, host_layer, x_all, seconds, threads):
    """Times the reference's CPU path on growing token samples until one takes
    about `seconds`; returns (tokens/s, tokens in the sample, seconds)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not O.ref_available():
        O.build(reference=False)
    rl = O.RefLayer(host_layer)
    n = 1
    while True:
        t0 = time.perf_counter()
        rl.forward(x_all[:n], threads=threads)
        dt = time.perf_counter() - t0
        if dt >= seconds or n >= x_all.shape[0]:
            return n / dt, n, dt
        n = min(x_all.shape[0], max(n + 1, int(n * min(8.0, 1.2 * seconds / max(dt, 1e-3)))))


def cpu_model() -> Optional[str]:
    """The host CPU's model name (/proc/cpuinfo), or None."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return None


def reference_arm(args, cfg, config, rank):
    """The reference's own CPU implementation of the layer (oracle/_ref: its
    CpuRouterBackend, CpuTensorBackend INT8 GEMMs and ExpertMlpExecutor
    compiled from its sources) on this host's cores.  Inputs come from the
    standalone build of the seeded generator, so libhmoe.so is never loaded
    in this process.  Rank 0 only."""
    import hmoe_api as H
    if rank != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    if not os.path.exists(O.SYNTH_PATH):
        O.build(reference=False)
    H.use_synth_library(O.SYNTH_PATH)
    T = args.tokens
    threads = os.cpu_count() or 1
    host_layer = H.make_host_layer(cfg, seed=args.seed)
    x = H.make_tokens(cfg, max(T, 1), seed=args.seed)
    per_step = max(1.0, min(6.0, 150.0 / max(1, args.steps + args.warmup)))
    rate, n, dt = cpu_reference_sample(cfg, host_layer, x, per_step, threads)
    rl = O.RefLayer(host_layer)
    for _ in range(args.warmup):
        rl.forward(x[:n], threads=threads)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        rl.forward(x[:n], threads=threads)
        times.append(time.perf_counter() - t0)
    value = n / statistics.mean(times)
    # the reference's own loop is single-threaded by construction
    # (CpuTensorBackend.cpp:173-186): one thread on a smaller sample
    rate1, n1, dt1 = cpu_reference_sample(cfg, host_layer, x, min(per_step, 5.0), 1)
    sample = (f"{n} of the {T} tokens per step (reference MoERuntime CPU branch: CpuRouterBackend + "
              f"CpuTensorBackend INT8 GEMMs; aggregate over {threads} host threads, one expert group per "
              f"thread at a time)")
    print(json.dumps({
        "metric": metric_for(args.config), "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * statistics.mean(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights quantised to INT8)",
        "config": config,
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "sample": sample,
                         "cpu_model": cpu_model()},
        "single_thread": {"value": rate1, "unit": UNIT, "cores": 1,
                          "sample": f"{n1} tokens in {dt1:.1f} s on one thread (the reference's own loop)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def config_subprocess(extra, timeout):
    """Another BASELINE configuration measured by this script in a process of
    its own, so that the c3 line's own figures never depend on it; returns
    that run's JSON line or why it is missing."""
    cmd = [sys.executable, os.path.abspath(__file__)] + extra
    env = {k: v for k, v in os.environ.items() if k not in ("RANK", "WORLD_SIZE", "LOCAL_RANK")}
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"`bench.py {' '.join(extra)}` did not finish within {timeout} s"}
    lines = [ln for ln in p.stdout.strip().splitlines() if ln.startswith("{")]
    if p.returncode != 0 or not lines:
        return {"unavailable": f"`bench.py {' '.join(extra)}` exited {p.returncode}: {p.stderr.strip()[-300:]}"}
    out = json.loads(lines[-1])
    out["command"] = " ".join(["python", "bench.py"] + extra)
    return out


def stack_subprocess(seed, steps, warmup, timeout=420):
    """the 48-block stack (prefill and decode)."""
    return config_subprocess(["--config", "c4", "--steps", str(steps), "--warmup", str(warmup),
                              "--seed", str(seed)], timeout)


def layer_subprocesses(seed, steps, warmup, timeout=300):
    """BASELINE configs[1] and [4] as single layers: C2 (Qwen1.5-MoE-A2.7B,
    shared experts) at its 512-token prefill and 1-token decode, and C5
    (Qwen3-235B-A22B) at 8192 tokens with 1- and 128-token decode batches.
    Device timing and stage splits only (no e2e, CPU or reference runs)."""
    common = ["--steps", str(steps), "--warmup", str(warmup), "--seed", str(seed), "--no-cpu-baseline",
              "--no-reference-cuda", "--no-e2e", "--no-stack"]
    return {"c2_t512": config_subprocess(["--config", "c2", "--tokens", "512", "--decode-tokens", "1"] + common,
                                         timeout),
            "c5_t8192": config_subprocess(["--config", "c5", "--tokens", "8192", "--decode-tokens", "1,128"] + common,
                                          timeout)}


def reference_cuda(cfg, T, seed, steps, warmup, gpu_index, pci, timeout=600):
    """Times the reference's own CUDA path (oracle/_ref/ref_cuda_bench: its
    CudaRouterBackend, per-expert gatherRows, ExpertMlpExecutor on
    CudaTensorBackend with planInt8Gemm's Auto mode, scatterAddRows) on this
    GPU, in a process of its own, with its own clock record.  Same seeded
    layer and tokens as the measured workload."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as O
    exe = O.REF_CUDA_BENCH
    if not os.path.exists(exe):
        return {"unavailable": "oracle/_ref/ref_cuda_bench is not built (needs the reference sources)"}
    cmd = [exe, "--hidden", str(cfg.hidden), "--inter", str(cfg.intermediate), "--experts", str(cfg.experts),
           "--topk", str(cfg.top_k), "--softmax", str(int(cfg.softmax)), "--renorm", str(int(cfg.renormalize)),
           "--shared", str(cfg.shared_experts), "--zipf", str(cfg.zipf_alpha or 0), "--tokens", str(T),
           "--seed", str(seed), "--steps", str(steps), "--warmup", str(warmup)]
    clocks = Clocks(gpu_index, pci)
    clocks.start()
    try:
        p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout)
    except subprocess.TimeoutExpired:
        clocks.stop()
        return {"unavailable": f"reference CUDA path did not finish within {timeout} s"}
    clk = clocks.stop()
    if p.returncode != 0:
        return {"unavailable": f"ref_cuda_bench exited {p.returncode}: {p.stderr.strip()[-300:]}"}
    out = json.loads(p.stdout.strip().splitlines()[-1])
    out["unit"] = UNIT
    out["clocks"] = clk
    out["timing"] = "wall clock per step (the path synchronises with the device inside each step), median"
    return out


def decode_split(layer, cfg, T, seed, dev, flush, events, peaks, steps=20):
    """Device-timed stage split of a decode-sized batch of T tokens on the
    resident layer: a CUDA-graph replay per step with the library's stage
    events, the L2 flushed before each step (a decode step touches fewer
    expert bytes than the L2 holds)."""
    import ctypes
    import numpy as np
    import torch
    import hmoe_api as H
    x = torch.from_numpy(H.make_tokens(cfg, T, seed=seed + 31)).to(dev)
    y = torch.empty_like(x)
    _, _, off, _, _ = layer.route(x)
    torch.cuda.synchronize()
    U = int((np.diff(off.cpu().numpy()) > 0).sum()) + cfg.shared_experts
    arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in events])

    def replay(variant):
        H.set_variant(variant)
        H.check("stage events", H.lib().hmoe_set_stage_events(arr, 6))
        try:
            for _ in range(3):
                layer.forward(x, y)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                layer.forward(x, y)
            torch.cuda.current_stream().wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                layer.forward(x, y)
            torch.cuda.synchronize()
            st = {s_: [] for s_ in STAGES}
            tot = []
            for _ in range(steps):
                flush.zero_()
                graph.replay()
                events[5].synchronize()
                tot.append(events[0].elapsed_time(events[5]))
                for i, s_ in enumerate(STAGES):
                    st[s_].append(events[i].elapsed_time(events[i + 1]))
            del graph
        finally:
            H.check("stage events", H.lib().hmoe_set_stage_events(None, 0))
            H.set_variant(0)
        return statistics.median(tot), {k: statistics.median(v) for k, v in st.items()}

    # The automatic choice (what a caller gets), the single-kernel decode
    # layer forced (it takes up to 8 tokens), the multi-kernel GEMV path
    # with its stage split and the multi-kernel tensor-core GEMM path.
    refused = {}

    def forced(variant, name):
        # a forced variant the shape or batch does not fit is reported, not fatal
        try:
            return replay(variant)
        except H.HmoeError as exc:
            refused[name] = str(exc)
            return None, None

    ms, med = replay(0)
    single_ms, _ = forced(3, "single_kernel") if T <= 8 else (None, None)
    multi_ms, multi = forced(1, "multi_kernel_gemv")
    gemm_ms, gemm = forced(2, "gemm")
    alg = algorithmic(cfg, T, U)
    roof_ms = 1e3 * max(alg["layer"]["bytes"] / (peaks["hbm_gbs"] * 1e9),
                        alg["layer"]["flops"] / (peaks["bf16_tflops"] * 1e12))
    expert_bytes = alg["gate_up"]["bytes"] + alg["down"]["bytes"]
    # expert bytes over the expert stages of the multi-kernel path, and over
    # the whole single-kernel layer (a lower bound of its expert stream rate)
    multi_expert_ms = multi["gate_up"] + multi["down"] if multi else None
    return {"tokens": T, "ms_per_step": ms, "value": T / (ms * 1e-3), "unit": UNIT,
            "single_kernel_ms": single_ms, "multi_kernel_ms": multi_ms, "multi_kernel_stages_ms": multi,
            "gemm_ms": gemm_ms, "gemm_stages_ms": gemm, "stages_ms": med,
            "variants_refused": refused or None,
            "unique_experts": U, "layer_roofline_ms": roof_ms,
            "layer_roofline_frac": roof_ms / ms,
            "expert_hbm_gbs": expert_bytes / (multi_expert_ms * 1e-3) / 1e9 if multi_expert_ms else None,
            "expert_hbm_frac": (expert_bytes / (multi_expert_ms * 1e-3) / 1e9 / peaks["hbm_gbs"]
                                if multi_expert_ms else None),
            "single_kernel_layer_hbm_frac": (alg["layer"]["bytes"] / (single_ms * 1e-3) / 1e9 / peaks["hbm_gbs"]
                                             if single_ms else None),
            "timing": "cuda-graph replay, median of %d steps, 256 MiB L2 flush before each" % steps}


STACK_METRIC = "MoE-stack tokens/s (Qwen3-30B-A3B, {layers} INT8 MoE layers)"


def reference_stack_sample(cfg, layers, seed, n, threads, repeats=1):
    """The reference's CPU path (oracle/_ref: its RMSNorm and MoE layer
    classes) through a stack of `layers` blocks, x += layer(rms_norm(x) * g)
    in FP32 as TransformerBlock::execute does with an identity attention, on
    `n` tokens.  Layers are generated from (seed, layer) one at a time
    (untimed); each block is run `repeats` times on the same input, so
    repeat r's stack time is the sum over blocks of the r-th run.  Returns
    the per-repeat seconds."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np
    import hmoe_api as H
    import oracle as O
    if not O.ref_available():
        O.build(reference=False)
    x = H.make_tokens(cfg, n, seed=seed)
    spent = [0.0] * repeats
    for l in range(layers):
        rl = O.RefLayer(H.make_host_layer(cfg, seed=seed, layer=l))
        g = H.make_norm_weight(cfg, seed, l)
        for r in range(repeats):
            t0 = time.perf_counter()
            y = rl.forward(O.rms_norm_ref(x, g, 1e-6), threads=threads)
            spent[r] += time.perf_counter() - t0
        x = (x + y).astype(np.float32)
        del rl
    return spent


def stack_main(args, world, rank, local):
    """the Qwen3-30B-A3B stack of 48 c3 MoE layers,
    weights per layer from (seed, layer), every layer resident (no tiering).
    Each block is hmoe_rms_norm then hmoe_moe_forward_residual in place
    (x += layer(rms_norm(x) * g), TransformerBlock::execute with an identity
    attention); over torchrun ranks hmoe_ep_moe_forward_residual with the routed experts
    split contiguously (16 per GPU at 8 ranks), one communicator and one
    registered workspace for the whole stack.  A step is a prefill of
    `--tokens` tokens per GPU through every layer (`value`, whole job); the
    `decode` object is a step of the `--decode-batch` batch (over all GPUs)
    through every layer."""
    import numpy as np
    import hmoe_api as H
    cfg = H.CONFIGS["c3"]
    L, T = args.layers, args.tokens
    Td = max(1, args.decode_batch // world)
    config = {"workload": f"c4: qwen3-30b-a3b {L}-layer moe stack (c3 layers)", "layers": L,
              "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k, "intermediate": cfg.intermediate,
              "prefill_tokens_per_gpu": T, "decode_batch": Td * world, "decode_tokens_per_gpu": Td,
              "routing": "zipf1.1 (bias per layer from seed+layer)", "weights": "int8 per-projection affine",
              "seed": args.seed, "parallelism": (f"ep{world}" if world > 1 else "single"),
              "ep_path": (args.ep_path if world > 1 else None),
              "placement": ("contiguous" if world > 1 else None),
              "l2": "inputs larger than L2 (the stack's INT8 experts), no flush"}
    threads = os.cpu_count() or 1
    if args.impl == "reference":
        if rank != 0:
            return
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if not os.path.exists(O.SYNTH_PATH):
            O.build(reference=False)
        H.use_synth_library(O.SYNTH_PATH)
        n = args.stack_cpu_tokens
        times = reference_stack_sample(cfg, L, args.seed, n, threads, repeats=max(1, args.steps))
        value = n / statistics.mean(times)
        print(json.dumps({
            "metric": STACK_METRIC.format(layers=L), "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": len(times), "warmup": 0, "ms_per_step": 1e3 * statistics.mean(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "fp32",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights quantised to INT8)",
            "config": config,
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "reference",
                             "sample": f"{n} tokens through all {L} layers per step, each layer run once per "
                                       f"step on the same input (layer generation untimed)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}))
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = comm = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        uid = [H.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = H.EpComm(uid[0], rank, world, timeout_ms=120000)
    H.set_variant(args.variant)
    H.set_route_variant(args.route_variant)

    # the reference CPU stack runs on a few tokens while the layers upload
    cpu = None
    cpu_on = world == 1 and not args.no_cpu_baseline
    spent = [0.0]
    if cpu_on:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle as O
        if not O.ref_available():
            O.build(reference=False)
    x_cpu = [H.make_tokens(cfg, args.stack_cpu_tokens, seed=args.seed)]

    def hosts():
        # each layer is generated once and used by both the device upload
        # and, on one GPU, the CPU sample
        for l in range(L):
            host = H.make_host_layer(cfg, seed=args.seed, layer=l)
            if cpu_on:
                rl = O.RefLayer(host)
                g = H.make_norm_weight(cfg, args.seed, l)
                t0 = time.perf_counter()
                y = rl.forward(O.rms_norm_ref(x_cpu[0], g, 1e-6), threads=threads)
                spent[0] += time.perf_counter() - t0
                x_cpu[0] = (x_cpu[0] + y).astype(np.float32)
                del rl
            yield host

    stack = H.MoEStack(cfg, L, seed=args.seed, device=dev, comm=comm, peer=args.ep_path == "peer", hosts=hosts())
    if cpu_on:
        n = args.stack_cpu_tokens
        cpu = {"value": n / spent[0], "unit": UNIT, "cores": threads, "kind": "reference",
               "sample": f"{n} tokens through all {L} blocks (RMSNorm + MoE layer) of the reference CPU path "
                         f"(oracle/_ref), "
                         f"{spent[0]:.1f} s in the layers, expert groups over {threads} threads"}

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    stream = torch.cuda.current_stream()

    def phase(Tn, seed_off, with_e2e):
        x0 = torch.from_numpy(H.make_tokens(cfg, Tn, seed=args.seed + seed_off + 7919 * rank)).to(dev)
        x = torch.empty_like(x0)

        def fwd():
            stack.forward(x, max_tokens=Tn)

        for _ in range(args.warmup):  # also sizes (and registers) the shared workspace
            x.copy_(x0)
            fwd()
        barrier()
        graph = None
        per = None
        if comm is None and not args.eager:
            side = torch.cuda.Stream()
            side.wait_stream(stream)
            with torch.cuda.stream(side):
                x.copy_(x0)
                fwd()
            stream.wait_stream(side)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            c1 = H.lib().hmoe_launch_count()
            with torch.cuda.graph(graph):
                fwd()
            per = H.lib().hmoe_launch_count() - c1
            torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        launches0 = H.lib().hmoe_launch_count()
        times = []
        barrier()
        for _ in range(args.steps):
            x.copy_(x0)
            e0.record(stream)
            if graph is not None:
                graph.replay()
            else:
                fwd()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        barrier()
        launches = per * args.steps if graph is not None else H.lib().hmoe_launch_count() - launches0
        ms = statistics.mean(times)
        e2e = None
        if with_e2e:
            xh = x0.cpu().pin_memory()
            yh = torch.empty_like(xh).pin_memory()
            et = []
            for i in range(args.steps + 1):
                barrier()
                e0.record(stream)
                x.copy_(xh, non_blocking=True)
                if graph is not None:
                    graph.replay()
                else:
                    fwd()
                yh.copy_(x, non_blocking=True)
                e1.record(stream)
                e1.synchronize()
                if i:
                    et.append(e0.elapsed_time(e1))
            em = statistics.mean(et)
            if dist is not None:
                t = torch.tensor([em], device=dev)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                em = float(t.item())
            e2e = {"value": world * Tn / (em * 1e-3), "unit": UNIT, "h2d_bytes_per_step": int(xh.numel() * 4),
                   "d2h_bytes_per_step": int(yh.numel() * 4), "ms_per_step": em,
                   "timing": "H2D copy of the step's tokens from page-locked memory, the stack, D2H copy of "
                             "its output; CUDA events on the launch stream"}
        if dist is not None:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        del graph
        return ms, launches, e2e

    props = torch.cuda.get_device_properties(dev)
    pci = None
    if hasattr(props, "pci_bus_id"):
        pci = f"{getattr(props, 'pci_domain_id', 0):08X}:{props.pci_bus_id:02X}:{getattr(props, 'pci_device_id', 0):02X}.0"
    clocks = Clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                    if os.environ.get("CUDA_VISIBLE_DEVICES") else local, pci)
    clocks.start()
    ms, launches, e2e = phase(T, 0, True)
    clk = clocks.stop()
    dms, dlaunches, _ = phase(Td, 31, False)
    status = stack.read_status()
    if rank == 0:
        peaks = load_peaks()
        # tensor-bound: router logits plus the routed rows' expert MLPs,
        # per GPU per layer (rows averaged over the ranks)
        flops = L * (2 * T * cfg.hidden * cfg.experts + 6 * T * cfg.top_k * cfg.hidden * cfg.intermediate)
        ach = flops / (ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "achieved": ach, "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                "frac": ach / peaks["bf16_tflops"], "kernel": "whole stack (all kernels of every layer)",
                "peak_source": peaks["source"] + " burst", "traffic": None}
        print(json.dumps({
            "metric": STACK_METRIC.format(layers=L), "value": world * T / (ms * 1e-3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "fp16+bf16",
            "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights quantised to INT8)",
            "config": config, "e2e": e2e, "gpu_launches": launches,
            "timing": ("cuda-graph replay of the stack (hmoe_rms_norm + hmoe_moe_forward_residual per layer)"
                       if comm is None else "eager hmoe_rms_norm + hmoe_ep_moe_forward_residual per layer"),
            "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
            "decode": {"tokens_per_step": Td * world, "ms_per_step": dms,
                       "value": Td * world / (dms * 1e-3), "unit": UNIT, "gpu_launches": dlaunches},
            "device_status": {"status": status[0], "near_ties": status[1], "sequential_logits": status[2]}}))
    if dist is not None:
        dist.barrier()
        comm.close()
        dist.destroy_process_group()


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.config == "c4":
        args.tokens = args.tokens or 2048
        stack_main(args, world, rank, local)
        return
    args.tokens = args.tokens or 4096
    import numpy as np
    import hmoe_api as H

    cfg = H.CONFIGS[args.config]
    T = args.tokens
    config = {"workload": WORKLOADS.get(args.config, args.config),
              "hidden": cfg.hidden, "experts": cfg.experts, "top_k": cfg.top_k,
              "intermediate": cfg.intermediate, "shared_experts": cfg.shared_experts,
              "tokens_per_gpu": T, "routing": "zipf1.1" if cfg.zipf_alpha else "uniform",
              "weights": "int8 per-projection affine", "seed": args.seed,
              "parallelism": (f"ep{world}" if world > 1 else "single"),
              "ep_path": (args.ep_path if world > 1 else None),
              "placement": (None if world == 1 else
                            "balanced from 4096 calibration tokens (seed+104729)" if args.placement == "balanced"
                            else "contiguous"),
              "l2": "inputs larger than L2 (INT8 expert arena) and a 256 MiB flush between steps"}

    if args.impl == "reference":
        reference_arm(args, cfg, config, rank)
        return

    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    comm = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=dev)
    H.set_variant(args.variant)
    H.set_route_variant(args.route_variant)
    host_layer = H.make_host_layer(cfg, seed=args.seed)
    x_np = H.make_tokens(cfg, T, seed=args.seed + 7919 * rank)
    if world > 1:
        # expert parallelism: this rank holds its contiguous share of the
        # routed experts; tokens stay on their rank (weak scaling)
        uid = [H.ep_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        comm = H.EpComm(uid[0], rank, world, timeout_ms=120000)
        placement = [None]
        if args.placement == "balanced" and rank == 0:
            # expert loads observed on a calibration batch (different seed
            # from every timed batch), routed on this GPU
            cal = H.DeviceLayer(host_layer, dev)
            xc = torch.from_numpy(H.make_tokens(cfg, 4096, seed=args.seed + 104729)).to(dev)
            _, _, off, _, _ = cal.route(xc)
            load = np.diff(off.cpu().numpy()).astype(np.float64)
            placement = [H.ep_balanced_placement(load, world)]
            del cal, xc
            torch.cuda.empty_cache()
        if args.placement == "balanced":
            dist.broadcast_object_list(placement, src=0)
        layer = H.EpLayer(host_layer, comm, dev, slot_of_expert=placement[0], peer=args.ep_path == "peer")
    else:
        layer = H.DeviceLayer(host_layer, dev)
    x = torch.from_numpy(x_np).to(dev)
    y = torch.empty_like(x)

    def forward():
        if comm is not None:
            layer.forward(x, y, max_tokens=T)
        else:
            layer.forward(x, y)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
    for e in ev:  # torch creates the CUDA event on first record
        e.record(stream)
    torch.cuda.synchronize()
    import ctypes
    arr = (ctypes.c_void_p * 6)(*[e.cuda_event for e in ev])

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()

    for _ in range(args.warmup):
        forward()
    barrier()

    # routing facts for the algorithmic byte/FLOP counts
    if comm is None:
        _, _, offsets, _, _ = layer.route(x)
        torch.cuda.synchronize()
        counts = np.diff(offsets.cpu().numpy())
        alg = algorithmic(cfg, T, int((counts > 0).sum()) + cfg.shared_experts)
    else:
        plan = comm.last_plan()
        rows_in = int(plan.recv_total) + T * cfg.shared_experts
        # every local expert counted as touched (an upper bound on the bytes)
        alg = algorithmic(cfg, T, int(plan.local_experts) + cfg.shared_experts, rows_in)
        alg["rows_received"] = int(plan.recv_total)
        # bytes this rank moves over NVLink per call: its dispatched rows (FP16
        # row + scale + routing weight) out and the outputs of the rows it
        # computed for other ranks (BF16) back out; the mirror image in
        row_out, row_ret = 2 * cfg.hidden + 8, 2 * cfg.hidden
        peers = [q for q in range(world) if q != rank]
        nv_out = sum(int(plan.send_rows[q]) * row_out + int(plan.recv_rows[q]) * row_ret for q in peers)
        nv_in = sum(int(plan.recv_rows[q]) * row_out + int(plan.send_rows[q]) * row_ret for q in peers)

    # Single GPU: one layer call, stage events included, captured once into a
    # CUDA graph (hmoe_moe_forward allocates nothing and never synchronises,
    # so it is capturable for a fixed token count); each timed step replays
    # it.  Expert parallelism reads the exchanged counts on the host once per
    # call, so it runs eagerly.
    H.check("stage events", H.lib().hmoe_set_stage_events(arr, 6))
    graph = None
    per_forward = None
    if not args.eager and comm is None:
        side = torch.cuda.Stream()
        side.wait_stream(stream)
        with torch.cuda.stream(side):
            forward()  # warm the side stream (attributes, tensor maps)
        stream.wait_stream(side)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        c1 = H.lib().hmoe_launch_count()
        with torch.cuda.graph(graph):
            forward()
        per_forward = H.lib().hmoe_launch_count() - c1
        torch.cuda.synchronize()
        stream = torch.cuda.current_stream()
    launches0 = H.lib().hmoe_launch_count()
    props = torch.cuda.get_device_properties(dev)
    pci = None
    if hasattr(props, "pci_bus_id"):
        pci = f"{getattr(props, 'pci_domain_id', 0):08X}:{props.pci_bus_id:02X}:{getattr(props, 'pci_device_id', 0):02X}.0"
    clocks = Clocks(int(os.environ.get("CUDA_VISIBLE_DEVICES", str(local)).split(",")[local])
                    if os.environ.get("CUDA_VISIBLE_DEVICES") else local, pci)
    clocks.start()
    stage_ms = {s: [] for s in STAGES}
    step_ms = []
    barrier()
    for _ in range(args.steps):
        flush.zero_()
        if graph is not None:
            graph.replay()
        else:
            forward()
        ev[5].synchronize()
        step_ms.append(ev[0].elapsed_time(ev[5]))
        for i, s in enumerate(STAGES):
            stage_ms[s].append(ev[i].elapsed_time(ev[i + 1]))
    barrier()
    clk = clocks.stop()
    launches = H.lib().hmoe_launch_count() - launches0
    if graph is not None:
        launches = per_forward * args.steps  # kernels inside each replayed graph
    H.check("stage events", H.lib().hmoe_set_stage_events(None, 0))
    ms = statistics.mean(step_ms)
    nvlink = None
    if dist is not None:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        nv = torch.tensor([float(nv_out), float(nv_in)], dtype=torch.float64, device=dev)
        nv_max = nv.clone()
        dist.all_reduce(nv_max, op=dist.ReduceOp.MAX)
        dist.all_reduce(nv, op=dist.ReduceOp.SUM)
        nvlink = {"bytes_out_per_rank_max": int(nv_max[0].item()), "bytes_in_per_rank_max": int(nv_max[1].item()),
                  "bytes_total": int(nv[0].item()),
                  "gbs_out_per_rank_max": nv_max[0].item() / (ms * 1e-3) / 1e9,
                  "gbs_in_per_rank_max": nv_max[1].item() / (ms * 1e-3) / 1e9,
                  "note": "per layer call: dispatched rows (FP16 + scale + weight) and returned outputs (BF16) "
                          "between different ranks, over the step time; link reference 770 GB/s per direction "
                          "(measured peer copy)"}
    value = world * T / (ms * 1e-3)

    # e2e: host buffers in and out, both copies inside the timed region
    # (single GPU: hmoe_moe_forward_host; expert parallelism: pinned copies
    # around hmoe_ep_moe_forward on the same stream)
    e2e = e2e_serial = None
    if not args.no_e2e:
        xh = torch.from_numpy(x_np).pin_memory()
        yh = torch.empty_like(xh).pin_memory()

        def forward_host():
            if comm is None:
                layer.forward_host(xh, yh)
            else:
                x.copy_(xh, non_blocking=True)
                layer.forward(x, y, max_tokens=T)
                yh.copy_(y, non_blocking=True)

        for _ in range(max(1, args.warmup // 2)):
            forward_host()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e2e_ms = []
        for _ in range(args.steps):
            flush.zero_()
            e0.record(stream)
            forward_host()
            e1.record(stream)
            e1.synchronize()
            e2e_ms.append(e0.elapsed_time(e1))
        em = statistics.mean(e2e_ms)
        if dist is not None:
            t = torch.tensor([em], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            em = float(t.item())
        e2e_serial = {"value": world * T / (em * 1e-3), "unit": UNIT, "h2d_bytes_per_step": int(x_np.nbytes),
                      "d2h_bytes_per_step": int(x_np.nbytes),
                      "timing": "one call at a time: 256 MiB L2 flush, then H2D copy, layer, D2H copy; CUDA events"}
        e2e = e2e_serial
        if comm is None:
            # A caller with a stream of batches keeps several calls in flight:
            # one stream, one workspace and one pair of page-locked buffers per
            # call in flight.  Each step still copies its own tokens in and its
            # output back; a call runs copy-in, layer, copy-out in order on its
            # stream, so with three in flight one call's layer overlaps the
            # others' copies in both directions.  The K steps are timed as a
            # whole (events on the first stream, the others joined into it).
            inflight = 3
            xhs, yhs = [xh], [yh]
            for i in range(1, inflight):
                xhs.append(torch.from_numpy(H.make_tokens(cfg, T, seed=args.seed + i)).pin_memory())
                yhs.append(torch.empty_like(xh).pin_memory())
            pstreams = [torch.cuda.Stream(device=dev) for _ in range(inflight)]
            pws = [torch.empty(layer.workspace_bytes(T, host_io=True), dtype=torch.uint8, device=dev)
                   for _ in range(inflight)]

            def pipelined(n):
                for i in range(n):
                    j = i % inflight
                    layer.forward_host(xhs[j], yhs[j], stream=pstreams[j], workspace=pws[j])

            pipelined(max(inflight, args.warmup))
            torch.cuda.synchronize()
            p0, p1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            p0.record(pstreams[0])
            for ps in pstreams[1:]:
                ps.wait_event(p0)
            pipelined(args.steps)
            for ps in pstreams[1:]:
                join = torch.cuda.Event()
                join.record(ps)
                pstreams[0].wait_event(join)
            p1.record(pstreams[0])
            p1.synchronize()
            pm = p0.elapsed_time(p1) / args.steps
            e2e = {"value": T / (pm * 1e-3), "unit": UNIT, "h2d_bytes_per_step": int(x_np.nbytes),
                   "d2h_bytes_per_step": int(x_np.nbytes), "ms_per_step": pm,
                   "timing": (f"{args.steps} hmoe_moe_forward_host calls, {inflight} in flight on {inflight} streams "
                              f"with {inflight} workspaces (each call: H2D copy of its tokens, layer, D2H copy of "
                              "its output); total time over the calls; inputs larger than L2 (INT8 expert arena), "
                              "no flush")}
            del pws

    status = layer.read_status()
    if rank != 0:
        if dist is not None:
            dist.barrier()
            comm.close()
            dist.destroy_process_group()
        return

    peaks = load_peaks()
    avg = {s: statistics.mean(v) for s, v in stage_ms.items()}
    top = max(STAGES, key=lambda s: avg[s])
    a = alg[top]
    dt_s = avg[top] * 1e-3
    if world == 1 and launches == args.steps:
        # one launch per step: the single-kernel decode layer runs the whole
        # layer, so its bytes are the layer's and its time the step's
        top, a, dt_s = "decode_layer", alg["layer"], ms * 1e-3
    ridge = peaks["bf16_tflops"] * 1e12 / (peaks["hbm_gbs"] * 1e9)
    tensor = a["flops"] > 0 and a["flops"] / max(a["bytes"], 1) > ridge
    if tensor:
        roof = {"bound": "tensor", "achieved": a["flops"] / dt_s / 1e12, "peak": peaks["bf16_tflops"],
                "unit": "TFLOP/s"}
    else:
        roof = {"bound": "hbm", "achieved": a["bytes"] / dt_s / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s"}
    roof["frac"] = roof["achieved"] / roof["peak"]
    roof["kernel"] = top
    roof["peak_source"] = peaks["source"] + (" burst" if tensor else "")
    roof["traffic"] = None
    tr_path = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tr_path):
        with open(tr_path) as f:
            tr = json.load(f)
        key = f"{args.config}:T{T}:{top}"
        if key in tr:
            roof["traffic"] = tr[key]["bytes_per_launch"]
    layer_roof_ms = 1e3 * max(alg["layer"]["bytes"] / (peaks["hbm_gbs"] * 1e9),
                              alg["layer"]["flops"] / (peaks["bf16_tflops"] * 1e12))

    cpu = None
    if not args.no_cpu_baseline and world == 1:
        threads = os.cpu_count() or 1
        rate, n, dt = cpu_reference_sample(cfg, host_layer, x_np, args.cpu_seconds, threads)
        cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "reference",
               "sample": f"{n} tokens of this workload through the reference CPU path "
                         f"(oracle/_ref), {dt:.1f} s, expert groups over {threads} threads",
               "cpu_model": cpu_model()}
        # the reference's own loop is single-threaded (CpuTensorBackend.cpp:173-186)
        rate1, n1, dt1 = cpu_reference_sample(cfg, host_layer, x_np, min(args.cpu_seconds, 5.0), 1)
        cpu["single_thread"] = {"value": rate1, "unit": UNIT, "cores": 1,
                                "sample": f"{n1} tokens in {dt1:.1f} s on one thread"}

    decode = None
    if world == 1 and T > 16 and not args.no_decode:
        decode = [decode_split(layer, cfg, t, args.seed, dev, flush, ev, peaks)
                  for t in (int(v) for v in args.decode_tokens.split(","))]

    ref_cuda = None
    ref_cuda_decode = None
    if world == 1 and not args.no_reference_cuda:
        gpu_index = clocks.index
        ref_cuda = reference_cuda(cfg, T, args.seed, 5, 2, gpu_index, pci)
        if T > 1:
            ref_cuda_decode = reference_cuda(cfg, 1, args.seed, 20, 3, gpu_index, pci)

    stack = others = None
    if world == 1 and args.config == "c3" and not args.no_stack:
        stack = stack_subprocess(args.seed, steps=5, warmup=3)
        others = layer_subprocesses(args.seed, steps=10, warmup=3)

    # tensor-core GEMM present (hmoe_set_variant(2) is refused without it)?
    has_gemm = H.lib().hmoe_set_variant(2) == 0
    H.lib().hmoe_set_variant(args.variant)
    used_gemm = has_gemm and args.variant != 1 and T * (cfg.top_k + cfg.shared_experts) > 64
    line = {
        "metric": metric_for(args.config),
        "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32" if not used_gemm else "fp16+bf16",
        "data": "synthetic (seeded N(0,1) activations, N(0,0.02^2) weights quantised to INT8)",
        "config": config,
        "e2e": e2e, "e2e_serial": e2e_serial, "gpu_launches": launches,
        "timing": ("cuda-graph replay of hmoe_moe_forward" if graph is not None else
                   "eager hmoe_ep_moe_forward" if comm is not None else "eager hmoe_moe_forward"),
        "roofline": roof, "cpu_baseline": cpu, "clocks": clk,
        "stages_ms": avg, "layer_roofline_ms": layer_roof_ms,
        "layer_roofline_frac": layer_roof_ms / ms, "unique_experts": alg["unique_experts"],
        "rows_received_rank0": alg.get("rows_received"),
        "nvlink": nvlink,
        "device_status": {"status": status[0], "near_ties": status[1], "sequential_logits": status[2]},
        "decode": decode,
        "reference_cuda": ref_cuda,
        "reference_cuda_decode_t1": ref_cuda_decode,
        "stack_c4": stack,
        "other_configs": others,
    }
    print(json.dumps(line))
    if dist is not None:
        dist.barrier()
        comm.close()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
