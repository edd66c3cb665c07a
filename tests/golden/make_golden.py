"""Generates tests/golden/*.npz from the reference's own CPU implementation.

Run in a container that has the reference sources (oracle/_ref is built from
them by oracle/Makefile):

    python tests/golden/make_golden.py

Every expected output below comes from oracle/_ref/libhmoe_ref.so, i.e. the
unmodified reference classes (CpuRouterBackend, CpuTensorBackend,
ExpertMlpExecutor, quantizeInt8) driven by oracle/ref_harness.cpp.  Large
inputs (expert arenas) are not stored: they are regenerated from their seed
by the synthetic generator and pinned by a SHA-256 recorded here, so the
fixtures stay small.  Deterministic inputs that the reference's own tests use
are reproduced from the formulas those tests state:

  tests/phase23_tests.cpp:189-201  INT8 GEMM shapes, x=(i%29-14)/29,
                                   q=((i*13)%255)-127, scale 0.003, zp -3
  tests/phase23_tests.cpp:305-321  INT8 MLP 1x513 -> 67 -> 513,
                                   x=(i%17-8)/17, scale 0.001, zp 0
  tests/phase22_tests.cpp:164-170  quantizer values {-2,-0.25,0,0.75,2}
  tests/phase12_tests.cpp:253-270  3-token / 3-expert top-2 routing
  tests/phase18_19_tests.cpp:233-263 router, gather, scatter vectors
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "hypermoe-engine_b200"))

import hmoe_api as H  # noqa: E402
import oracle as O  # noqa: E402

OUT = os.path.dirname(os.path.abspath(__file__))


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def phase23_inputs(rows, inner, cols):
    i = np.arange(rows * inner)
    x = ((i % 29) - 14).astype(np.float32) / np.float32(29.0)
    j = np.arange(inner * cols)
    q = (((j * 13) % 255) - 127).astype(np.int8)
    return x.reshape(rows, inner), q.reshape(inner, cols)


GEMM_SHAPES = [(1, 8, 8), (1, 257, 65), (2, 513, 33), (1, 1031, 31), (1, 2048, 768),
               (1, 768, 2048), (3, 129, 7), (1, 4097, 67)]


def gen_gemm():
    R = O.ref()
    d = {}
    for (r, k, n) in GEMM_SHAPES:
        x, q = phase23_inputs(r, k, n)
        d[f"out_{r}_{k}_{n}"] = O.int8_matmul(R, x, q, np.float32(0.003), -3)
    np.savez_compressed(os.path.join(OUT, "int8_gemm_phase23.npz"), **d)


def gen_mlp():
    R = O.ref()
    i = np.arange(513)
    x = (((i % 17) - 8).astype(np.float32) / np.float32(17.0)).reshape(1, 513)

    def qmat(rows, cols):
        j = np.arange(rows * cols)
        return (((j * 13) % 255) - 127).astype(np.int8).reshape(rows, cols)

    g, u, dn = qmat(513, 67), qmat(513, 67), qmat(67, 513)
    y = O.expert_mlp(R, x, g, u, dn, np.full(3, 0.001, np.float32), np.zeros(3, np.int32))
    np.savez_compressed(os.path.join(OUT, "int8_mlp_phase23.npz"), x=x, y=y)


def gen_quant():
    R = O.ref()
    vals = np.array([-2.0, -0.25, 0.0, 0.75, 2.0], np.float32)
    q, s, z, e = O.quantize(R, vals)
    rng = np.random.default_rng(7)
    w = (rng.standard_normal(4099) * 0.02).astype(np.float32)
    q2, s2, z2, e2 = O.quantize(R, w)
    np.savez_compressed(os.path.join(OUT, "quantize.npz"), vals=vals, q=q, scale=s, zp=z, err=e,
                        w=w, q2=q2, scale2=s2, zp2=z2, err2=e2)


def gen_router():
    R = O.ref()
    rng = np.random.default_rng(11)
    cases = {}
    for name, (T, Hd, E, k, sm, rn, bias) in {
        "a": (33, 64, 60, 4, True, False, False),
        "b": (17, 96, 128, 8, True, True, True),
        "c": (9, 32, 8, 2, False, True, False),
        "d": (20, 128, 256, 8, True, True, True),
    }.items():
        x = rng.standard_normal((T, Hd)).astype(np.float32)
        w = (rng.standard_normal((Hd, E)) * 0.02).astype(np.float32)
        b = H.synth_zipf_bias(5, 1.1, E) if bias else None
        ids, sc, off, gt, gs = O.route(R, x, w, b, k, sm, rn)
        cases.update({f"{name}_x": x, f"{name}_w": w, f"{name}_ids": ids, f"{name}_scores": sc,
                      f"{name}_offsets": off, f"{name}_gtok": gt, f"{name}_gsc": gs,
                      f"{name}_cfg": np.array([T, Hd, E, k, int(sm), int(rn), int(bias)], np.int64)})
        if b is not None:
            cases[f"{name}_bias"] = b
    # Reference KATs: phase12 (3 tokens, 2 hidden, 3 experts, top-2) and
    # phase18_19 (same router matrix shape, different hidden).
    x12 = np.array([[1, 0], [0, 1], [1, 1]], np.float32)
    w12 = np.array([[3, 2, 0], [0, 2, 3]], np.float32)
    ids, sc, off, gt, gs = O.route(R, x12, w12, None, 2, True, True)
    cases.update(p12_x=x12, p12_w=w12, p12_ids=ids, p12_scores=sc, p12_offsets=off, p12_gtok=gt)
    x18 = np.array([[-2, -1], [0, 1], [2, 3]], np.float32)
    w18 = np.array([[2, 0, 1], [0, 2, 1]], np.float32)
    ids, sc, off, gt, gs = O.route(R, x18, w18, None, 2, True, True)
    cases.update(p18_x=x18, p18_w=w18, p18_ids=ids, p18_scores=sc)
    np.savez_compressed(os.path.join(OUT, "router.npz"), **cases)


def gen_layer(name, cfg_key, T, seed):
    cfg = H.CONFIGS[cfg_key]
    hl = H.make_host_layer(cfg, seed=seed)
    x = H.make_tokens(cfg, T, seed=seed)
    rl = O.RefLayer(hl)
    out, ids, sc, off = rl.forward(x, threads=os.cpu_count() or 1, want_routing=True)
    np.savez_compressed(
        os.path.join(OUT, f"layer_{name}.npz"), out=out, ids=ids, scores=sc, offsets=off,
        meta=np.array([T, seed], np.int64),
        sha_x=np.array(sha(x)), sha_router=np.array(sha(hl.router_w)), sha_arena=np.array(sha(hl.arena)),
        sha_bias=np.array(sha(hl.router_bias) if hl.router_bias is not None else ""),
        scales=hl.scales, zps=hl.zps)


def main():
    O.build(reference=True)
    gen_gemm()
    gen_mlp()
    gen_quant()
    gen_router()
    gen_layer("c1_t64", "c1", 64, 0)
    gen_layer("c3_t16", "c3", 16, 0)
    gen_layer("c2_t3", "c2", 3, 1)
    gen_layer("c5_t4", "c5", 4, 2)
    for f in sorted(os.listdir(OUT)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(OUT, f)))


if __name__ == "__main__":
    main()
