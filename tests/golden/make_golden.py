"""Generates the golden fixtures in this directory from the reference itself.

Runs the reference's own C sources (oracle/_ref/libkmamba_ref.so, built in
place from the k-mamba tree by oracle/Makefile) on seeded inputs and saves
inputs + outputs as small .npz files:

  scan1d_bwd.npz   cpu/scan1d_backward.c        (shapes of tests/unit/test_scan1d_backward.c)
  scannd.npz       src/scan_nd.c scannd_ref     (shapes of tests/test_cuda_scan_nd.cu)
  convnd.npz       src/convnd.c convnd()        forward + backward, 1D/2D/3D
  plans.npz        src/wavefront_plan.c         level_starts / level_offsets

The 1D/2D forward kernels of the reference are NASM (not buildable here);
they are pinned in the tests by the reference tests' own known answers.

Run from the repository root:  python tests/golden/make_golden.py
(needs the reference tree at build time only; the fixtures travel).
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "k-mamba_b200"))
os.environ.setdefault("OMP_NUM_THREADS", "1")  # scannd_ref races under OpenMP

import oracle  # noqa: E402
import kmamba_b200 as kb  # noqa: E402  (struct layouts are the reference's)

OUT = os.path.dirname(os.path.abspath(__file__))
f32 = np.float32


def P(a):
    return a.ctypes.data


def gen_scan1d_bwd(ref, rng):
    cases = {}
    for (L, D, M) in [(4, 8, 1), (8, 16, 1), (4, 8, 2), (8, 16, 2), (33, 5, 3), (64, 24, 16)]:
        x = rng.uniform(-1, 1, (L, D)).astype(f32)
        A = rng.uniform(-1, -0.01, (D, M)).astype(f32)
        B = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
        Cm = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
        dt = rng.uniform(0.01, 0.5, (L, D)).astype(f32)
        dy = rng.uniform(-1, 1, (L, D)).astype(f32)
        h0 = rng.uniform(-0.5, 0.5, (D, M)).astype(f32)
        _, _, h_all = oracle.scan1d_fwd(x, dt, A, B, Cm, h0=h0, clamp=False, want_h_all=True)
        outs = {k: np.zeros(s, f32) for k, s in
                [("dx", (L, D)), ("dA", (D, M)), ("dB", (L, D, M)), ("dC", (L, D, M)),
                 ("ddelta", (L, D))]}
        p = kb.ScanBackwardParams(P(x), P(A), P(B), P(Cm), P(dt), P(h0), P(h_all), P(dy),
                                  P(outs["dx"]), P(outs["dA"]), P(outs["dB"]), P(outs["dC"]),
                                  P(outs["ddelta"]), L, D, M)
        ref.scan1d_backward(C.byref(p))
        tag = f"{L}x{D}x{M}"
        for k, v in dict(x=x, A=A, B=B, C=Cm, dt=dt, dy=dy, h0=h0, h=h_all, **outs).items():
            cases[f"{tag}/{k}"] = v
    np.savez_compressed(os.path.join(OUT, "scan1d_bwd.npz"), **cases)


def gen_scannd(ref, rng):
    cases = {}
    for dims, D, M in [((8,), 3, 2), ((3, 4), 2, 3), ((2, 2, 3), 2, 2), ((5, 7), 4, 4),
                       ((3, 4, 5), 3, 2), ((2, 3, 2, 3), 2, 3)]:
        dims_a = np.array(dims, np.int64)
        nd = len(dims)
        Pn = int(np.prod(dims))
        x = rng.uniform(-1, 1, (Pn, D)).astype(f32)
        A = rng.uniform(-1.0, -0.05, (nd, D, M)).astype(f32)
        B = rng.uniform(-0.5, 0.5, (Pn, D, M)).astype(f32)
        Cm = rng.uniform(-0.5, 0.5, (Pn, D, M)).astype(f32)
        delta = rng.uniform(0.01, 0.3, (nd, Pn, D)).astype(f32)
        h = np.zeros((Pn, D, M), f32)
        y = np.zeros((Pn, D), f32)
        p = kb.ScanNDParams(P(dims_a), nd, D, M, P(x), P(A), P(B), P(Cm), P(delta), P(h), P(y),
                            None, None)
        ref.scannd_ref.argtypes = [C.POINTER(kb.ScanNDParams)]
        rc = ref.scannd_ref(C.byref(p))
        assert rc == 0
        tag = "x".join(map(str, dims)) + f"_D{D}_M{M}"
        for k, v in dict(dims=dims_a, x=x, A=A, B=B, C=Cm, delta=delta, h=h, y=y).items():
            cases[f"{tag}/{k}"] = v
    np.savez_compressed(os.path.join(OUT, "scannd.npz"), **cases)


def gen_convnd(ref, rng):
    cases = {}
    ref.convnd.argtypes = [C.POINTER(kb.ConvNDParams), C.c_int]
    for dims, D, K in [((9,), 3, 3), ((2, 2), 1, 2), ((6, 5), 4, 3), ((4, 3, 5), 2, 2),
                       ((7, 6), 5, 4), ((3, 3, 3), 3, 3)]:
        dims_a = np.array(dims, np.int64)
        nd = len(dims)
        Pn = int(np.prod(dims))
        KV = K ** nd
        inp = rng.normal(0, 1, (Pn, D)).astype(f32)
        ker = rng.normal(0, 1.0 / 3, (KV, D)).astype(f32)
        bias = rng.normal(0, 0.1, (D,)).astype(f32)
        dy = rng.normal(0, 1, (Pn, D)).astype(f32)
        out = np.zeros((Pn, D), f32)
        din = np.zeros((Pn, D), f32)
        dk = np.zeros((KV, D), f32)
        db = np.zeros((D,), f32)
        p = kb.ConvNDParams(P(inp), P(ker), P(bias), P(out), P(dy), P(din), P(dk), P(db),
                            P(dims_a), nd, D, K)
        ref.convnd(C.byref(p), 3)
        tag = "x".join(map(str, dims)) + f"_D{D}_K{K}"
        for k, v in dict(dims=dims_a, input=inp, kernel=ker, bias=bias, dy=dy, output=out,
                         dinput=din, dkernel=dk, dbias=db).items():
            cases[f"{tag}/{k}"] = v
    np.savez_compressed(os.path.join(OUT, "convnd.npz"), **cases)


def gen_plans(ref):
    cases = {}
    ref.km_wavefront_plan_create.restype = C.POINTER(kb.KMWavefrontPlan)
    ref.km_wavefront_plan_create.argtypes = [C.c_void_p, C.c_long]
    ref.km_wavefront_plan_free.argtypes = [C.POINTER(kb.KMWavefrontPlan)]
    for dims in [(1,), (7,), (3, 4), (2, 3, 2), (5, 1, 4), (4, 4, 4), (2, 3, 4, 5),
                 (1, 1, 1, 1, 6), (16, 16), (2, 2, 2, 2, 2, 2, 2, 2)]:
        dims_a = np.array(dims, np.int64)
        pl = ref.km_wavefront_plan_create(P(dims_a), len(dims)).contents
        nl = pl.max_level + 2
        tag = "x".join(map(str, dims))
        cases[f"{tag}/dims"] = dims_a
        cases[f"{tag}/level_starts"] = np.ctypeslib.as_array(pl.level_starts, (nl,)).copy()
        cases[f"{tag}/level_offsets"] = np.ctypeslib.as_array(pl.level_offsets,
                                                              (pl.total_points,)).copy()
        cases[f"{tag}/meta"] = np.array([pl.total_points, pl.max_level, pl.max_level_size],
                                        np.int64)
        ref.km_wavefront_plan_free(C.pointer(pl))
    np.savez_compressed(os.path.join(OUT, "plans.npz"), **cases)


def main():
    oracle.build()
    ref = oracle.ref_lib()
    if ref is None:
        sys.exit("oracle/_ref/libkmamba_ref.so missing: build it with `make -C oracle` "
                 "where the reference tree is available")
    rng = np.random.default_rng(20261201)
    gen_scan1d_bwd(ref, rng)
    gen_scannd(ref, rng)
    gen_convnd(ref, rng)
    gen_plans(ref)
    print("golden fixtures written to", OUT)


if __name__ == "__main__":
    main()
