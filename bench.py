#!/usr/bin/env python3
"""Benchmark of the k-mamba hot path on B200 (one JSON line on rank 0).

Workload ("config 2"): 1D selective scan forward
+ backward in fp32, batch 8, L 4096, D 1536, N 16, B/C shared across
channels, synthetic inputs with the config's distributions.  One step =
kmb_scan1d_fwd (y + checkpoints) then kmb_scan1d_bwd (dx, ddt, dA, dB, dC).

metric: algorithmic HBM GB/s of the step (bytes a perfect kernel must
move: fwd 4(3E + 2BLN + DN), bwd 4(5E + 4BLN + 2DN), E = B*L*D) divided by
the device time.  Every [B,L,D] tensor is 201 MB, larger than the 126 MB
L2, so no flush is needed between steps.

--impl reference times the reference's own CPU implementation of the path
(oracle/_ref: src/scan_nd.c scannd_ref for the forward states and
cpu/scan1d_backward.c for the backward) on the host cores, on bounded
samples of the same workload, with the same metric.

Multi-GPU (torchrun): every rank runs a full config-2 batch of its own
(weak scaling), or with --shard-batch the config's batch of 8 is split over
the ranks (strong scaling).  The only exchange is the sum of the parameter
gradient dA over ranks, all-reduced by the library's own NCCL communicator
(kmamba_distributed.h) on a side stream while the next forward runs.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "k-mamba_b200"))

BATCH, L, D, N = 8, 4096, 1536, 16
E = BATCH * L * D
FWD_BYTES = 4 * (3 * E + 2 * BATCH * L * N + D * N)
BWD_BYTES = 4 * (5 * E + 4 * BATCH * L * N + 2 * D * N)
STEP_BYTES = FWD_BYTES + BWD_BYTES


def set_batch(b):
    global BATCH, E, FWD_BYTES, BWD_BYTES, STEP_BYTES
    BATCH = b
    E = BATCH * L * D
    FWD_BYTES = 4 * (3 * E + 2 * BATCH * L * N + D * N)
    BWD_BYTES = 4 * (5 * E + 4 * BATCH * L * N + 2 * D * N)
    STEP_BYTES = FWD_BYTES + BWD_BYTES


WORKLOAD = ("config2: 1D selective scan fwd+bwd, fp32, batch 8, L 4096, D 1536, N 16, "
            "B/C shared across D")
METRIC = "scan HBM GB/s (algorithmic bytes / device time), 1D selective scan fwd+bwd"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


def make_inputs(seed, batch=None, d=D):
    """Config-2 distributions: x, dy ~ N(0,1); dt = softplus(N(0,1) - 2);
    A = -exp(U[ln 1, ln 16]); B, C ~ N(0,1) of shape (B, L, N)."""
    batch = BATCH if batch is None else batch
    rng = np.random.default_rng(seed)
    f = np.float32
    x = rng.standard_normal((batch, L, d), dtype=f)
    dt = np.log1p(np.exp(rng.standard_normal((batch, L, d), dtype=f) - 2)).astype(f)
    A = (-np.exp(rng.uniform(0, np.log(16), (d, N)))).astype(f)
    B = rng.standard_normal((batch, L, N), dtype=f)
    Cm = rng.standard_normal((batch, L, N), dtype=f)
    dy = rng.standard_normal((batch, L, d), dtype=f)
    return x, dt, A, B, Cm, dy


class Clocks:
    """Samples nvidia-smi during the timed region."""

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        d = os.environ.get("KMB_CLOCKS_DIR") or tempfile.gettempdir()
        os.makedirs(d, exist_ok=True)
        self.path = os.path.join(d, f"clocks_gpu{self.index}.csv")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.index)],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            self.proc.wait()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 7:
                continue
            try:
                rows.append((float(parts[0]), float(parts[1]), float(parts[2]), parts[3:]))
            except ValueError:
                continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3])
                          if v.lower().startswith("active")})
        loaded = [r for r in rows if r[2] > 250] or rows
        return {"sm_mhz": statistics.median(r[0] for r in loaded),
                "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows),
                "samples": len(rows), "reasons": reasons}


def traffic_from_profile():
    """DRAM bytes per launch of the dominant kernel from the committed ncu
    summary (profiles/scan1d_config2_traffic.json), if present."""
    p = os.path.join(ROOT, "profiles", "scan1d_config2_traffic.json")
    try:
        with open(p) as f:
            return json.load(f)
    except (OSError, ValueError):
        return None


# --------------------------------------------------------------------------
# reference CPU arm / CPU baseline
# --------------------------------------------------------------------------

CPU_SLICES, CPU_CHANS = 96, 16  # one batch item: 96 slices x 16 channels = D


def cpu_bench_lib():
    """The OpenMP driver of the reference's own CPU path (oracle/_ref,
    kind "reference"), or of its C restatement when the reference build is
    absent (kind "port").  Test infrastructure: bench.py's CPU legs only."""
    ref = os.path.join(ROOT, "oracle", "_ref", "libkmb_refbench.so")
    if os.path.exists(ref):
        lib, kind = C.CDLL(ref), "reference"
    else:
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import oracle  # noqa: WPS433  (CPU baseline leg only)
        if not os.path.exists(oracle.ORACLE_SO):
            oracle.build()
        lib, kind = C.CDLL(oracle.ORACLE_SO), "port"
    lib.kmb_cpu_bench_create.restype = C.c_void_p
    lib.kmb_cpu_bench_create.argtypes = [C.c_int, C.c_int, C.c_long, C.c_int, C.c_ulonglong,
                                         C.c_int]
    lib.kmb_cpu_bench_pass.restype = C.c_double
    lib.kmb_cpu_bench_pass.argtypes = [C.c_void_p]
    lib.kmb_cpu_bench_free.argtypes = [C.c_void_p]
    return lib, kind


def cpu_sample_desc(nth):
    return (f"one of the {BATCH} batch items per step: all {D} channels as "
            f"{CPU_SLICES} slices x {CPU_CHANS} channels, full L={L}, N={N}, B/C expanded to "
            f"the reference's [L,D,N] layout; reference scannd_ref (ndims 1) forward + "
            f"scan1d_backward per slice under one OpenMP parallel loop on {nth} host threads "
            f"(one thread-local reference pool per OpenMP worker); inputs pre-touched by "
            f"their worker outside the timed region")


def cpu_reference_run(nth, warmup, steps, seed=1):
    """Seconds per pass (mean of `steps` timed passes after `warmup`) of the
    reference's CPU path over one batch item of config 2.  Returns
    (seconds, channel_sequences, kind)."""
    lib, kind = cpu_bench_lib()
    h = lib.kmb_cpu_bench_create(CPU_SLICES, CPU_CHANS, L, N, seed, nth)
    if not h:
        raise RuntimeError("CPU baseline: host allocation failed")
    try:
        for _ in range(warmup):
            lib.kmb_cpu_bench_pass(h)
        secs = [lib.kmb_cpu_bench_pass(h) for _ in range(max(1, steps))]
    finally:
        lib.kmb_cpu_bench_free(h)
    return sum(secs) / len(secs), CPU_SLICES * CPU_CHANS, kind


def cpu_threads():
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 96))


def bytes_for_channels(nch):
    return STEP_BYTES * nch / (BATCH * D)


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    nth = cpu_threads()
    t, nch, kind = cpu_reference_run(nth, args.warmup, args.steps, seed=100)
    v = bytes_for_channels(nch) / t / 1e9
    sample = cpu_sample_desc(nth)
    line = {"metric": METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t * 1e3 * BATCH * D / nch,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "batch": BATCH, "L": L, "D": D, "N": N,
                       "ms_per_sampled_pass": t * 1e3},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": nth, "kind": kind,
                             "sample": sample},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# secondary workloads (configs 3 and 4), single GPU, device-resident
# --------------------------------------------------------------------------

def lib_comm(lib, kb, dist, world, rank, local):
    """The library's own NCCL communicator (kmamba_distributed.h); its
    unique id travels over torch.distributed.  None for one rank."""
    if world <= 1:
        return None
    uid = C.create_string_buffer(128)
    if rank == 0:
        kb.check(lib, lib.kmb_dist_get_unique_id(uid))
    box = [uid.raw if rank == 0 else None]
    dist.broadcast_object_list(box, src=0)
    ctx = lib.kmb_dist_init_with_id(world, rank, local, C.create_string_buffer(box[0], 128))
    if not ctx:
        raise RuntimeError(kb.last_error(lib))
    return ctx


def run_secondary(args):
    """Times one forward + backward of BASELINE config 3 (ConvND 512x512,
    D 64, K 3, batch 16) or config 4 (2D scan 256x256, batch 8, D 256,
    N 16, B/C shared, same dt on both axes) and prints one JSON line with
    the per-kernel roofline.  Algorithmic bytes: inputs read once plus
    outputs written once.

    Under torchrun every rank runs the same pass on its share of the
    config's batch (--shard-batch: the batch split over the ranks, the
    fixed-batch series; otherwise a full batch per rank), and the
    parameter gradients (dkernel / dbias, or dA) are summed over the ranks
    by the library's NCCL communicator after every backward.  Time: max
    over ranks; value: bytes of all ranks per second."""
    import torch
    import torch.distributed as dist
    import kmamba_b200 as kb
    import kmb_dist
    rank, world = kmb_dist.env_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        kmb_dist.init("nccl", timeout_s=120, device_id=torch.device("cuda", local))
    lib = kb.load()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    lib.kmb_set_stream(sp)
    lib.kmb_set_sync(0)
    ctx = lib_comm(lib, kb, dist, world, rank, local)

    def share(full):
        """(items on this rank, items of the whole job)"""
        if args.batch is not None:
            return args.batch, args.batch * world
        if args.shard_batch and world > 1:
            n = full // world + (1 if rank < full % world else 0)
            if n == 0:
                raise SystemExit(f"--shard-batch: {world} ranks for a batch of {full}")
            return n, full
        return full, full * world
    f = np.float32
    rng = np.random.default_rng(kmb_dist.shard_seed(7, rank))
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, dtype=f)).cuda()  # noqa: E731
    dtype = "f32"
    if args.workload == "conv3":
        (bsz, gbatch), H, W, Dc, K = share(16), 512, 512, 64, 3
        Pn = H * W
        E3 = bsz * Pn * Dc
        # activations (input, output, dy, dinput) in fp32 or bf16; taps,
        # bias and their gradients fp32
        ab = 2 if args.io == "bf16" else 4
        fwd_b, bwd_b = ab * 2 * E3 + 4 * 640, ab * 3 * E3 + 4 * 1280
        scale_job = gbatch / bsz
        act = (lambda a: dev(a).to(torch.bfloat16)) if ab == 2 else dev
        inp = act(rng.standard_normal((bsz, Pn, Dc), dtype=f))
        ker = dev(rng.standard_normal((9, Dc), dtype=f) / 3)
        bias = dev(rng.standard_normal((Dc,), dtype=f) * 0.1)
        dy = act(rng.standard_normal((bsz, Pn, Dc), dtype=f))
        out, din = torch.empty_like(inp), torch.empty_like(inp)
        dk, db = torch.empty_like(ker), torch.empty_like(bias)
        a = kb.KmbConvND()
        a.input, a.kernel, a.bias, a.output = (t.data_ptr() for t in (inp, ker, bias, out))
        a.dy, a.dinput, a.dkernel, a.dbias = (t.data_ptr() for t in (dy, din, dk, db))
        a.dims[0], a.dims[1] = H, W
        a.ndims, a.batch, a.D, a.K = 2, bsz, Dc, K
        ffn, bfn = ((lib.kmb_convnd_fwd_bf16, lib.kmb_convnd_bwd_bf16) if ab == 2
                    else (lib.kmb_convnd_fwd, lib.kmb_convnd_bwd))
        fwd = lambda: kb.check(lib, ffn(C.byref(a)))  # noqa: E731
        bwd = lambda: kb.check(lib, bfn(C.byref(a)))  # noqa: E731
        names = ("k_conv2d_fwd_ring", "k_conv2d_bwd_ring")
        grads = [(dk, 9 * Dc), (db, Dc)]
        dtype = "bf16 I/O, fp32 math" if ab == 2 else "f32"
        workload = (f"config3: ConvND 2D 512x512, D 64, K 3, batch {gbatch} ({bsz} per GPU), "
                    f"{'bf16 activations' if ab == 2 else 'fp32'}, fwd+bwd")
        metric = "ConvND HBM GB/s (algorithmic bytes / device time)"
    else:
        (bsz, gbatch), H, W, Dc, Nn = share(8), 256, 256, 256, 16
        Pn = H * W
        E4 = bsz * Pn * Dc
        # bf16 I/O: x, dt, B, C, y, dy, dx, ddelta, dB, dC in 2 bytes; A, dA fp32
        ab = 2 if args.io == "bf16" else 4
        fwd_b = ab * (3 * E4 + 2 * bsz * Pn * Nn) + 4 * 2 * Dc * Nn
        bwd_b = ab * (5 * E4 + 4 * bsz * Pn * Nn) + 4 * 4 * Dc * Nn
        scale_job = gbatch / bsz
        act = (lambda a: dev(a).to(torch.bfloat16)) if ab == 2 else dev
        x = act(rng.standard_normal((bsz, Pn, Dc), dtype=f))
        dt1 = (np.log1p(np.exp(rng.standard_normal((bsz, 1, Pn, Dc), dtype=f) - 2)) +
               np.log(2)).astype(f)
        delta = act(np.concatenate([dt1, dt1], axis=1))  # same dt on both axes
        A = dev(-np.exp(rng.uniform(0, np.log(16), (2, Dc, Nn))))
        B = act(rng.standard_normal((bsz, Pn, Nn), dtype=f))
        Cm = act(rng.standard_normal((bsz, Pn, Nn), dtype=f))
        dy = act(rng.standard_normal((bsz, Pn, Dc), dtype=f))
        h = torch.empty((bsz, Pn, Dc, Nn), device="cuda")
        y, dx = torch.empty_like(x), torch.empty_like(x)
        ddl, dA = torch.empty_like(delta), torch.empty_like(A)
        dB, dC = torch.empty_like(B), torch.empty_like(Cm)

        class KmbScanND(C.Structure):
            _fields_ = [(n, C.c_void_p) for n in ("x", "delta", "A", "B", "C", "h", "y", "dy",
                                                  "dx", "ddelta", "dA", "dB", "dC")] + [
                ("dims", C.c_long * 8), ("ndims", C.c_long), ("batch", C.c_long),
                ("D", C.c_long), ("M", C.c_long), ("bc_shared", C.c_int), ("flags", C.c_int)]
        a = KmbScanND()
        a.x, a.delta, a.A, a.B, a.C, a.h, a.y = (t.data_ptr() for t in (x, delta, A, B, Cm, h, y))
        a.dy, a.dx, a.ddelta, a.dA, a.dB, a.dC = (t.data_ptr() for t in (dy, dx, ddl, dA, dB, dC))
        a.dims[0], a.dims[1] = H, W
        a.ndims, a.batch, a.D, a.M, a.bc_shared = 2, bsz, Dc, Nn, 1
        ffn, bfn = ((lib.kmb_scannd_fwd_bf16, lib.kmb_scannd_bwd_bf16) if ab == 2
                    else (lib.kmb_scannd_fwd, lib.kmb_scannd_bwd))
        ffn.argtypes = [C.c_void_p]
        bfn.argtypes = [C.c_void_p]
        fwd = lambda: kb.check(lib, ffn(C.byref(a)))  # noqa: E731
        bwd = lambda: kb.check(lib, bfn(C.byref(a)))  # noqa: E731
        dtype = "bf16 I/O, fp32 math and states" if ab == 2 else "f32"
        names = ("k_scan2d_fwd", "k_scan2d_bwd")
        grads = [(dA, 2 * Dc * Nn)]
        workload = (f"config4: 2D selective scan 256x256, batch {gbatch} ({bsz} per GPU), D 256, "
                    + ("N 16, bf16 tensors (fp32 A, dA, h), " if ab == 2 else "N 16, fp32, ")
                    + "B/C shared, dt = softplus(N(0,1)-2) + ln 2 on both axes, fwd+bwd "
                    "(stored-state kernels of the reference API)")
        metric = "scan HBM GB/s (algorithmic bytes / device time), 2D selective scan fwd+bwd"
    def exchange():
        # sum of the parameter gradients over the ranks (side stream,
        # ordered after the backward; the next step's backward waits)
        if ctx:
            for t, n in grads:
                kb.check(lib, lib.kmb_dist_bucket_add(ctx, t.data_ptr(), n, 0, sp))
            kb.check(lib, lib.kmb_dist_bucket_flush(ctx, sp))

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    for _ in range(args.warmup):
        fwd()
        if ctx:
            kb.check(lib, lib.kmb_dist_wait(ctx, sp))
        bwd()
        exchange()
    if ctx:
        kb.check(lib, lib.kmb_dist_wait(ctx, sp))
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    marks = [[ev(), ev(), ev()] for _ in range(args.steps)]
    start, stop = ev(), ev()
    with Clocks(local) as clk:
        start.record(stream)
        for m in marks:
            m[0].record(stream)
            fwd()
            if ctx:
                kb.check(lib, lib.kmb_dist_wait(ctx, sp))
            m[1].record(stream)
            bwd()
            m[2].record(stream)
            exchange()
        if ctx:
            kb.check(lib, lib.kmb_dist_wait(ctx, sp))
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed = kmb_dist.max_over_ranks(start.elapsed_time(stop) / 1e3, world, device="cuda")
    fms = sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps
    bms = sum(m[1].elapsed_time(m[2]) for m in marks) / args.steps
    pk, pk_kind = peaks()
    dom = (bms, bwd_b, names[1]) if bms >= fms else (fms, fwd_b, names[0])
    ach = dom[1] / (dom[0] / 1e3) / 1e9
    job_bytes = (fwd_b + bwd_b) * scale_job
    if ctx:
        lib.kmamba_distributed_fini_nccl(ctx)
    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    print(json.dumps({
        "metric": metric, "value": job_bytes * args.steps / elapsed / 1e9, "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if (args.shard_batch and world > 1) else "weak",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic", "config": {"workload": workload, "fwd_ms": fms, "bwd_ms": bms,
                                        "batch_per_gpu": bsz, "global_batch": gbatch,
                                        "parallelism": f"dp{world} (parameter gradients summed by "
                                                       "the library's NCCL communicator)",
                                        "fwd_GBps": fwd_b / fms / 1e6,
                                        "bwd_GBps": bwd_b / bms / 1e6},
        "roofline": {"bound": "hbm", "kernel": dom[2], "achieved": ach, "peak": pk["hbm_gbs"],
                     "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                     "peak_source": f"{pk_kind} hbm_gbs", "traffic": None},
        "gpu_launches": 2 * args.steps, "clocks": clk.summary()}), flush=True)
    if world > 1:
        dist.destroy_process_group()


# --------------------------------------------------------------------------
# tensor-core GEMM of the block projections (kmb_gemm_bf16)
# --------------------------------------------------------------------------

def run_gemm(args):
    """Times kmb_gemm_bf16 on the projection shapes of a dim-1024 Mamba-ND
    block: in_proj [T, 1024] x [2048, 1024]^T and
    out_proj [T, 1024] x [1024, 1024]^T with T = --gemm-m tokens, bf16
    operands and output, fp32 accumulation; plus the two gradient GEMMs of
    in_proj (MN-major operands).  Reports TFLOP/s against the measured
    cuBLAS bf16 peak."""
    import torch
    import kmamba_b200 as kb
    lib = kb.load()
    stream = torch.cuda.current_stream()
    lib.kmb_set_stream(C.c_void_p(stream.cuda_stream))
    lib.kmb_set_sync(0)
    T = args.gemm_m
    g = torch.Generator(device="cuda").manual_seed(1234)
    bf = torch.bfloat16
    x = torch.randn(T, 1024, device="cuda", generator=g).to(bf)
    w_in = (torch.randn(2048, 1024, device="cuda", generator=g) / 32).to(bf)
    w_out = (torch.randn(1024, 1024, device="cuda", generator=g) / 32).to(bf)
    z = torch.empty(T, 2048, device="cuda", dtype=bf)
    y = torch.empty(T, 1024, device="cuda", dtype=bf)
    dz = torch.randn(T, 2048, device="cuda", generator=g).to(bf)
    dx = torch.empty(T, 1024, device="cuda", dtype=bf)
    dw = torch.empty(2048, 1024, device="cuda", dtype=torch.float32)

    def mk(A, B, Cc, M, N, K, lda, ldb, ldc, amn=0, bmn=0, c16=1):
        a = kb.KmbGemm()
        a.A, a.B, a.C = A.data_ptr(), B.data_ptr(), Cc.data_ptr()
        a.M, a.N, a.K, a.lda, a.ldb, a.ldc = M, N, K, lda, ldb, ldc
        a.a_mn_major, a.b_mn_major, a.c_bf16 = amn, bmn, c16
        return a
    ops = [("in_proj", mk(x, w_in, z, T, 2048, 1024, 1024, 1024, 2048), 2 * T * 2048 * 1024),
           ("out_proj", mk(x, w_out, y, T, 1024, 1024, 1024, 1024, 1024), 2 * T * 1024 * 1024),
           # dx = dz W_in: A = dz [T, 2048] K-major, B = W_in^T: [1024, 2048] stored [2048, 1024]
           ("in_proj_dx", mk(dz, w_in, dx, T, 1024, 2048, 2048, 1024, 1024, 0, 1),
            2 * T * 1024 * 2048),
           # dW = dz^T x: A = dz^T [2048, T] stored [T, 2048], B = x^T [1024, T] stored [T, 1024]
           ("in_proj_dw", mk(dz, x, dw, 2048, 1024, T, 2048, 1024, 1024, 1, 1, 0),
            2 * T * 2048 * 1024)]
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    for _ in range(args.warmup):
        for _, a, _ in ops:
            kb.check(lib, lib.kmb_gemm_bf16(C.byref(a)))
    torch.cuda.synchronize()
    marks = [[ev() for _ in range(len(ops) + 1)] for _ in range(args.steps)]
    with Clocks(0) as clk:
        for m in marks:
            m[0].record(stream)
            for i, (_, a, _) in enumerate(ops):
                kb.check(lib, lib.kmb_gemm_bf16(C.byref(a)))
                m[i + 1].record(stream)
        torch.cuda.synchronize()
    kb.check(lib, lib.kmb_gemm_check_error())
    per = {name: sum(m[i].elapsed_time(m[i + 1]) for m in marks) / args.steps
           for i, (name, _, _) in enumerate(ops)}
    flops = sum(f for _, _, f in ops)
    ms = sum(per.values())
    pk, pk_kind = peaks()
    tf = {name: f / (per[name] / 1e3) / 1e12 for name, _, f in ops}
    dom = max(per, key=per.get)
    print(json.dumps({
        "metric": "bf16 GEMM TFLOP/s (block projections, tcgen05)", "value": flops / (ms / 1e3) / 1e12,
        "unit": "TFLOP/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "bf16", "data": "synthetic",
        "config": {"workload": f"dim-1024 block projections, T={T} tokens: in_proj, out_proj, "
                               "in_proj input and weight gradients",
                   **{k + "_ms": v for k, v in per.items()},
                   **{k + "_TFLOPs": v for k, v in tf.items()}},
        "roofline": {"bound": "tensor", "kernel": "k_gemm_tc (" + dom + ")",
                     "achieved": tf[dom], "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                     "frac": tf[dom] / pk["bf16_tflops"],
                     "peak_source": f"{pk_kind} bf16_tflops (cuBLAS burst)", "traffic": None},
        "gpu_launches": len(ops) * args.steps, "clocks": clk.summary()}), flush=True)


# --------------------------------------------------------------------------
# config 5 at kernel level: one Mamba-ND layer's ConvND + ND scan over 64^3
# --------------------------------------------------------------------------

def run_nd5(args):
    """Kernel-level stand-in for BASELINE config 5, whose 24-layer model is
    not built: one layer's causal depthwise ConvND (K 3) and 3-axis ND
    selective scan (N 16, B/C shared across channels, per-axis A and delta),
    forward and backward, over 64^3 volumes with dim channels (default
    1024), batch per GPU (default 1: the reference API's state history h and
    the backward's adjoint G are [P, D, N] each, 17 GB per item at dim
    1024).  Reports volume tokens per second of that layer; no projection
    GEMMs, gating or optimizer step are in the timed region."""
    import torch
    import kmamba_b200 as kb
    lib = kb.load()
    stream = torch.cuda.current_stream()
    lib.kmb_set_stream(C.c_void_p(stream.cuda_stream))
    lib.kmb_set_sync(0)
    bsz = args.batch or 1
    dims, Dc, Nn, K = [64, 64, 64], args.dim or 1024, 16, 3
    nd, Pn = 3, 64 ** 3
    g = torch.Generator(device="cuda").manual_seed(1234)
    rn = lambda *sh: torch.randn(*sh, device="cuda", generator=g)  # noqa: E731
    x = rn(bsz, Pn, Dc)
    delta = (torch.nn.functional.softplus(rn(bsz, nd, Pn, Dc) - 2) + float(np.log(3))).contiguous()
    A = -torch.exp(torch.rand(nd, Dc, Nn, device="cuda", generator=g) * float(np.log(16)))
    B, Cm, dy = rn(bsz, Pn, Nn), rn(bsz, Pn, Nn), rn(bsz, Pn, Dc)
    h = torch.empty((bsz, Pn, Dc, Nn), device="cuda")
    y, dx = torch.empty_like(x), torch.empty_like(x)
    ddl, dA, dB, dC = (torch.empty_like(t) for t in (delta, A, B, Cm))
    ker, bias = rn(K ** nd, Dc) / 5, rn(Dc) * 0.1
    cout, cdin = torch.empty_like(x), torch.empty_like(x)
    dk, db = torch.empty_like(ker), torch.empty_like(bias)

    class KmbScanND(C.Structure):
        _fields_ = [(n, C.c_void_p) for n in ("x", "delta", "A", "B", "C", "h", "y", "dy",
                                              "dx", "ddelta", "dA", "dB", "dC")] + [
            ("dims", C.c_long * 8), ("ndims", C.c_long), ("batch", C.c_long),
            ("D", C.c_long), ("M", C.c_long), ("bc_shared", C.c_int), ("flags", C.c_int)]
    a = KmbScanND()
    a.x, a.delta, a.A, a.B, a.C, a.h, a.y = (t.data_ptr() for t in (x, delta, A, B, Cm, h, y))
    a.dy, a.dx, a.ddelta, a.dA, a.dB, a.dC = (t.data_ptr() for t in (dy, dx, ddl, dA, dB, dC))
    for i, v in enumerate(dims):
        a.dims[i] = v
    a.ndims, a.batch, a.D, a.M, a.bc_shared = nd, bsz, Dc, Nn, 1
    lib.kmb_scannd_fwd.argtypes = [C.c_void_p]
    lib.kmb_scannd_bwd.argtypes = [C.c_void_p]
    c = kb.KmbConvND()
    c.input, c.kernel, c.bias, c.output = (t.data_ptr() for t in (x, ker, bias, cout))
    c.dy, c.dinput, c.dkernel, c.dbias = (t.data_ptr() for t in (dy, cdin, dk, db))
    for i, v in enumerate(dims):
        c.dims[i] = v
    c.ndims, c.batch, c.D, c.K = nd, bsz, Dc, K
    ops = (("conv_fwd", lambda: kb.check(lib, lib.kmb_convnd_fwd(C.byref(c)))),
           ("scan_fwd", lambda: kb.check(lib, lib.kmb_scannd_fwd(C.byref(a)))),
           ("scan_bwd", lambda: kb.check(lib, lib.kmb_scannd_bwd(C.byref(a)))),
           ("conv_bwd", lambda: kb.check(lib, lib.kmb_convnd_bwd(C.byref(c)))))
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    for _ in range(args.warmup):
        for _, f in ops:
            f()
    torch.cuda.synchronize()
    marks = [[ev() for _ in range(len(ops) + 1)] for _ in range(args.steps)]
    with Clocks(0) as clk:
        for m in marks:
            m[0].record(stream)
            for i, (_, f) in enumerate(ops):
                f()
                m[i + 1].record(stream)
        torch.cuda.synchronize()
    per = {name: sum(m[i].elapsed_time(m[i + 1]) for m in marks) / args.steps
           for i, (name, _) in enumerate(ops)}
    ms = sum(per.values())
    E = bsz * Pn * Dc
    hbytes = 4 * E * Nn
    print(json.dumps({
        "metric": "Mamba-ND layer tokens/s (kernel level: ConvND 3D + ND scan 3D, fwd+bwd)",
        "value": bsz * Pn / (ms / 1e3), "unit": "tokens/s", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"config5 kernels: 64^3 volume, dim {Dc}, N {Nn}, K {K}, "
                               f"batch {bsz}, B/C shared, fp32 (one layer's ConvND + ND scan; "
                               "the 24-layer model is not built)",
                   **{k + "_ms": v for k, v in per.items()},
                   "scan_mufu_bound_ms_per_pass": E * Nn * nd / (148 * 16 * 1.965e9) * 1e3,
                   "scan_state_history_GB": hbytes / 1e9},
        "gpu_launches": 6 * args.steps, "clocks": clk.summary()}), flush=True)


# --------------------------------------------------------------------------
# config 5: the Mamba-ND model (kmamba_ndmodel.h), tokens/s of a train step
# --------------------------------------------------------------------------

def run_nd5_model(args):
    """BASELINE config 5 through kmamba_ndmodel.h: 24 ND blocks (dim 1024,
    16 states, ConvND K 3) over 64^3 volumes of byte tokens (uniform in
    [0, 256), seeded per rank), fp32 masters with bf16 GEMMs, one
    kmb_ndmodel_train_step (forward, per-layer recompute + backward, NCCL
    average of the gradients when N > 1, AdamW) per step.  value = tokens
    of all ranks per second (max over ranks); e2e = the same with each
    step's tokens copied from pinned host memory and the loss read back.
    Batch per GPU defaults to BASELINE's 64 volumes over 8 GPUs = 8, run as
    micro-batches of as many volumes as fit (one at dim 1024: the
    stored-state ND scan keeps a [P, d, 16] history for the layer being
    differentiated, 17 GB per volume) whose gradients accumulate before the
    NCCL average and AdamW."""
    import torch
    import torch.distributed as dist
    import kmamba_b200 as kb
    import kmb_dist
    rank, world = kmb_dist.env_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        kmb_dist.init("nccl", timeout_s=300, device_id=torch.device("cuda", local))
    lib = kb.load()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    lib.kmb_set_stream(sp)
    lib.kmb_set_sync(0)
    dims = [args.nd_side] * 3
    P = int(np.prod(dims))
    bsz = args.batch or 8
    cfg = kb.KmbNDModelConfig()
    for i in range(3):
        cfg.dims[i] = dims[i]
    cfg.dim, cfg.n_layers, cfg.vocab, cfg.seed = args.dim or 1024, args.layers, 256, 1234
    m = lib.kmb_ndmodel_create(C.byref(cfg))
    if not m:
        raise RuntimeError(kb.last_error(lib))
    ctx = None
    if world > 1:
        uid = C.create_string_buffer(128)
        if rank == 0:
            kb.check(lib, lib.kmb_dist_get_unique_id(uid))
        box = [uid.raw if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ctx = lib.kmb_dist_init_with_id(world, rank, local, C.create_string_buffer(box[0], 128))
        if not ctx:
            raise RuntimeError(kb.last_error(lib))
        # identical initial weights on every rank (rank 0's)
        if lib.kmamba_broadcast_params_nccl(ctx, lib.kmb_ndmodel_params(m),
                                            lib.kmb_ndmodel_param_count(m)) != 0:
            raise RuntimeError(kb.last_error(lib))
        kb.check(lib, lib.kmb_ndmodel_sync_weights(m))
        kb.check(lib, lib.kmb_ndmodel_set_dist(m, ctx))
    rng = np.random.default_rng(kmb_dist.shard_seed(5000, rank))
    tok = rng.integers(0, 256, (bsz, P), dtype=np.uint32)
    dtok = torch.from_numpy(tok.astype(np.int32)).cuda()
    loss = C.c_float()
    lr, wd = 1e-4, 0.0

    def step(ptr):
        kb.check(lib, lib.kmb_ndmodel_train_step(m, ptr, bsz, lr, wd, C.byref(loss)))

    for _ in range(args.warmup):
        step(dtok.data_ptr())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731
    start, stop = ev(), ev()
    with Clocks(local) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step(dtok.data_ptr())
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed = kmb_dist.max_over_ranks(start.elapsed_time(stop) / 1e3, world, device="cuda")
    value = bsz * P * world * args.steps / elapsed
    # e2e: tokens from pinned host memory every step, loss read back
    htok = torch.from_numpy(tok.astype(np.int32)).pin_memory()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(max(1, args.e2e_steps)):
        step(htok.data_ptr())
    torch.cuda.synchronize()
    te = kmb_dist.max_over_ranks((time.perf_counter() - t0) / max(1, args.e2e_steps), world,
                                 device="cuda")
    if ctx:
        lib.kmamba_distributed_fini_nccl(ctx)
    lib.kmb_ndmodel_free(m)
    if rank == 0:
        # projection FLOPs of a step: forward a, z, out (3 d^2), the
        # backward's recompute of a, z (2 d^2) and its six gradient GEMMs
        # (6 d^2), per token and layer, x 2 FLOP per multiply-add
        gemm_flops = 2 * bsz * P * 11 * cfg.dim * cfg.dim * cfg.n_layers
        print(json.dumps({
            "metric": "Mamba-ND model train tokens/s (config 5)", "value": value,
            "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 GEMMs, fp32 scan / conv / masters",
            "data": "synthetic byte tokens, uniform in [0, 256), seeded per rank",
            "config": {"workload": f"config5: {cfg.n_layers} ND blocks, dim {cfg.dim}, 16 states, "
                                   f"ConvND K 3, {dims[0]}^3 volumes, batch {bsz} per GPU "
                                   f"(global {bsz * world}; BASELINE: 64 over 8 GPUs), "
                                   "micro-batches sized to the free memory",
                       "parallelism": f"dp{world}: kmamba_distributed.h NCCL buckets per layer, "
                                      "average, overlapped with the backward",
                       "loss": loss.value,
                       "projection_TFLOPs_per_gpu": gemm_flops * args.steps / elapsed / 1e12},
            "e2e": {"value": bsz * P * world / te, "unit": "tokens/s",
                    "h2d_bytes_per_step": 4 * bsz * P, "d2h_bytes_per_step": 4},
            "gpu_launches": None, "clocks": clk.summary()}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# --------------------------------------------------------------------------
# config 1: the README KMamba model through kmamba.h
# --------------------------------------------------------------------------

MODEL1_CFG = dict(vocab_size=256, dim=384, state_size=1024, seq_len=128, n_layers=1)
MODEL1_WORKLOAD = ("config1: KMamba LM (vocab 256, dim 384, state 1024, seq_len 128, 1 layer, "
                   "kmamba_init(1234), tokens srand(0) rand()%256), one kmamba_forward + one "
                   "kmamba_train_step per step, lr 1e-3, clip_norm 1.0, host token/logit "
                   "buffers through the C API")


def _model1(libm):
    """Builds the config-1 model with `libm` (ours or the reference's)."""
    import kmamba_b200 as kb
    cfg = kb.KMambaConfig()
    for k, v in MODEL1_CFG.items():
        setattr(cfg, k, v)
    m = libm.kmamba_create(C.byref(cfg))
    libm.kmamba_init(m, 1234)
    o = kb.MBOptimConfig()
    o.lr, o.clip_norm = 1e-3, 1.0
    libm.kmamba_enable_training(m, C.byref(o), 1e-3, 1e-5)
    libc = C.CDLL(None)
    libc.srand(0)
    toks = np.array([libc.rand() % 256 for _ in range(129)], dtype=np.uint32)
    logits = np.zeros(128 * 256, np.float32)
    return m, toks, logits


def _model1_step(libm, m, toks, logits):
    libm.kmamba_forward(m, toks.ctypes.data, logits.ctypes.data)
    return libm.kmamba_train_step(m, toks.ctypes.data)


def _model1_cpu(steps):
    """ms per step of the reference's own CPU build (oracle/_ref), all host
    threads (OpenMP inside its GEMMs)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as o
    import kmamba_b200 as kb
    ref = o.ref_lib()
    if ref is None:
        return None
    kb.declare(ref, kb.MODEL_PROTOTYPES)
    m, toks, logits = _model1(ref)
    _model1_step(ref, m, toks, logits)
    t0 = time.perf_counter()
    for _ in range(steps):
        _model1_step(ref, m, toks, logits)
    ms = (time.perf_counter() - t0) / steps * 1e3
    ref.kmamba_free(m)
    return ms


def run_model1(args):
    """Times config 1: one kmamba_forward + one kmamba_train_step per step
    through the C API with host buffers (the API's own contract: tokens and
    logits in host memory, weights and Adam moments in the host structs,
    staged to the device by every call).  value = ms per step, host wall
    clock around the synchronous calls; device_ms = CUDA-event time on the
    library stream over the same steps."""
    import torch
    import kmamba_b200 as kb
    lib = kb.load()
    stream = torch.cuda.current_stream()
    lib.kmb_set_stream(C.c_void_p(stream.cuda_stream))
    lib.kmb_set_sync(1)
    m, toks, logits = _model1(lib)
    for _ in range(args.warmup):
        _model1_step(lib, m, toks, logits)
    torch.cuda.synchronize()
    n0 = lib.kmb_block_launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(0) as clk:
        e0.record(stream)
        t0 = time.perf_counter()
        for _ in range(args.steps):
            _model1_step(lib, m, toks, logits)
        e1.record(stream)
        torch.cuda.synchronize()
        wall = (time.perf_counter() - t0) / args.steps * 1e3
    dev_ms = e0.elapsed_time(e1) / args.steps
    launches = lib.kmb_block_launch_count() - n0
    # the same steps with the model device-resident (kmamba_resident.h): no
    # per-call copies of weights, gradients and moments
    kb.check(lib, lib.kmamba_set_device_resident(m, 1))
    for _ in range(args.warmup):
        _model1_step(lib, m, toks, logits)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        _model1_step(lib, m, toks, logits)
    torch.cuda.synchronize()
    resident_ms = (time.perf_counter() - t0) / args.steps * 1e3
    kb.check(lib, lib.kmamba_set_device_resident(m, 0))
    lib.kmamba_free(m)
    cpu = None if args.no_cpu_baseline else _model1_cpu(3)
    V, L = 256, 128
    h2d = 4 * (129 + 129)  # tokens of forward + train_step (weights: see staged_bytes)
    print(json.dumps({
        "metric": "KMamba config-1 step time (kmamba_forward + kmamba_train_step)",
        "value": wall, "unit": "ms/step", "n_gpus": 1, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": wall, "higher_is_better": False,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": MODEL1_WORKLOAD, "device_ms_per_step": dev_ms,
                   "resident_ms_per_step": resident_ms,
                   "l2": "working set < L2 (the config is small); weights restaged per call "
                         "(resident_ms_per_step: the model made device-resident first)"},
        "e2e": {"value": wall, "unit": "ms/step", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": 4 * (L * V + L)},
        "cpu_baseline": None if cpu is None else {
            "value": cpu, "unit": "ms/step", "cores": os.cpu_count(), "kind": "reference",
            "sample": "3 steps of the same workload, reference CPU build (OpenMP)"},
        "gpu_launches": int(launches), "clocks": clk.summary()}), flush=True)


# --------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------

def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=None,
                    help="batch items per GPU (profiling of small cases only; default: "
                         "the workload's BASELINE batch)")
    ap.add_argument("--dim", type=int, default=None,
                    help="nd5 only: channels (default 1024; smaller for profiling captures)")
    ap.add_argument("--io", choices=["f32", "bf16"], default="f32",
                    help="conv3 / scan2d4: element type of the activation / scan tensors")
    ap.add_argument("--layers", type=int, default=24, help="nd5model only: ND blocks")
    ap.add_argument("--nd-side", type=int, default=64, help="nd5model only: volume side")
    ap.add_argument("--shard-batch", action="store_true",
                    help="scan1d: split the config's batch over the ranks (strong scaling) "
                         "instead of a full batch per rank (weak scaling, the default)")
    ap.add_argument("--gemm-m", type=int, default=32768,
                    help="gemm only: tokens (rows) of the projection GEMMs")
    ap.add_argument("--workload", default="scan1d",
                    choices=["scan1d", "conv3", "scan2d4", "model1", "nd5", "nd5model", "gemm"],
                    help="scan1d = BASELINE config 2 (the headline); conv3 / scan2d4 time "
                         "configs 3 and 4 for their roofline evidence")
    args = ap.parse_args()
    if args.batch is not None and args.workload == "scan1d":
        set_batch(args.batch)
    if args.impl == "reference":
        run_reference_arm(args)
        return
    if args.workload == "model1":
        run_model1(args)
        return
    if args.workload == "nd5":
        run_nd5(args)
        return
    if args.workload == "gemm":
        run_gemm(args)
        return
    if args.workload == "nd5model":
        run_nd5_model(args)
        return
    if args.workload != "scan1d":
        run_secondary(args)
        return

    import torch
    import torch.distributed as dist
    import kmamba_b200 as kb
    import kmb_dist

    rank, world = kmb_dist.env_rank()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    global_batch = BATCH
    if args.shard_batch:
        # strong scaling: the config's batch split over the ranks (earlier
        # ranks take the extra items, kmamba_distributed_split_batch's rule)
        set_batch(global_batch // world + (1 if rank < global_batch % world else 0))
        if BATCH == 0:
            raise SystemExit(f"--shard-batch: {world} ranks for a batch of {global_batch}")
    global_bytes = STEP_BYTES * global_batch / BATCH if args.shard_batch else STEP_BYTES * world
    if world > 1:
        kmb_dist.init("nccl", timeout_s=120, device_id=torch.device("cuda", local))
    lib = kb.load()
    stream = torch.cuda.current_stream()
    sp = C.c_void_p(stream.cuda_stream)
    lib.kmb_set_stream(sp)
    lib.kmb_set_sync(0)
    # the data-parallel exchange (dA) runs on the library's own NCCL
    # communicator; torch.distributed only carries its id, the barriers and
    # the max-over-ranks timing
    ctx = None
    if world > 1:
        uid = C.create_string_buffer(128)
        if rank == 0:
            kb.check(lib, lib.kmb_dist_get_unique_id(uid))
        box = [uid.raw if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        ctx = lib.kmb_dist_init_with_id(world, rank, local, C.create_string_buffer(box[0], 128))
        if not ctx:
            raise RuntimeError(kb.last_error(lib))

    x, dt, A, B, Cm, dy = make_inputs(seed=kmb_dist.shard_seed(1000, rank))
    dev = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    tx, tdt, tA, tB, tC, tdy = map(dev, (x, dt, A, B, Cm, dy))
    ty = torch.empty_like(tx)
    nck = lib.kmb_scan1d_ckpt_elems(BATCH, L, D, N)
    tck = torch.empty(nck, dtype=torch.float32, device="cuda")
    g = {k: torch.empty(s, dtype=torch.float32, device="cuda") for k, s in
         (("dx", (BATCH, L, D)), ("ddt", (BATCH, L, D)), ("dA", (D, N)),
          ("dB", (BATCH, L, N)), ("dC", (BATCH, L, N)))}

    fa = kb.KmbScan1D()
    fa.x, fa.dt, fa.A, fa.B, fa.C = (t.data_ptr() for t in (tx, tdt, tA, tB, tC))
    fa.y, fa.ckpt = ty.data_ptr(), tck.data_ptr()
    fa.batch, fa.L, fa.D, fa.N, fa.bc_shared, fa.clamp = BATCH, L, D, N, 1, 1
    ba = kb.KmbScan1D()
    C.memmove(C.byref(ba), C.byref(fa), C.sizeof(fa))
    ba.y = None
    ba.dy = tdy.data_ptr()
    ba.dx, ba.ddt, ba.dA, ba.dB, ba.dC = (g[k].data_ptr() for k in ("dx", "ddt", "dA", "dB", "dC"))

    ev = lambda: torch.cuda.Event(enable_timing=True)  # noqa: E731

    def step(marks=None):
        if marks:
            marks[0].record(stream)
        kb.check(lib, lib.kmb_scan1d_fwd(C.byref(fa)))
        if ctx:
            # the previous step's dA reduction (overlapped with this
            # forward) must end before this backward overwrites dA
            kb.check(lib, lib.kmb_dist_wait(ctx, sp))
        if marks:
            marks[1].record(stream)
        kb.check(lib, lib.kmb_scan1d_bwd(C.byref(ba)))
        if marks:
            marks[2].record(stream)
        if ctx:
            kb.check(lib, lib.kmb_dist_bucket_add(ctx, g["dA"].data_ptr(), D * N, 0, sp))
            kb.check(lib, lib.kmb_dist_bucket_flush(ctx, sp))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    marks = [[ev(), ev(), ev()] for _ in range(args.steps)]
    start, stop = ev(), ev()
    with Clocks(local) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(marks[i])
        if ctx:
            kb.check(lib, lib.kmb_dist_wait(ctx, sp))  # the last step's reduction
        stop.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    elapsed = start.elapsed_time(stop) / 1e3
    fwd_ms = sum(m[0].elapsed_time(m[1]) for m in marks) / args.steps
    bwd_ms = sum(m[1].elapsed_time(m[2]) for m in marks) / args.steps
    elapsed = kmb_dist.max_over_ranks(elapsed, world, device="cuda")
    value = global_bytes * args.steps / elapsed / 1e9

    # ---------------- e2e through the public C ABI with host buffers ----------
    h2d = d2h = 0
    e2e_val = None
    if args.e2e_steps > 0:
        pin = lambda a: torch.from_numpy(a).pin_memory()  # noqa: E731
        hx, hdt, hA, hB, hC, hdy = map(pin, (x, dt, A, B, Cm, dy))
        hy = torch.empty(x.shape, dtype=torch.float32).pin_memory()
        hg = {k: torch.empty(tuple(v.shape), dtype=torch.float32).pin_memory()
              for k, v in g.items()}
        ef = kb.KmbScan1D()
        ef.x, ef.dt, ef.A, ef.B, ef.C = (t.data_ptr() for t in (hx, hdt, hA, hB, hC))
        ef.y = hy.data_ptr()
        ef.batch, ef.L, ef.D, ef.N, ef.bc_shared, ef.clamp = BATCH, L, D, N, 1, 1
        eb = kb.KmbScan1D()
        C.memmove(C.byref(eb), C.byref(ef), C.sizeof(ef))
        eb.y = None
        eb.dy = hdy.data_ptr()
        eb.dx, eb.ddt, eb.dA, eb.dB, eb.dC = (hg[k].data_ptr()
                                              for k in ("dx", "ddt", "dA", "dB", "dC"))
        lib.kmb_set_sync(1)
        fin = [hx, hdt, hA, hB, hC]
        h2d = sum(t.numel() * 4 for t in fin) * 2 + hdy.numel() * 4
        d2h = hy.numel() * 4 + sum(t.numel() * 4 for t in hg.values())
        kb.check(lib, lib.kmb_scan1d_fwd(C.byref(ef)))  # warm the staging pool
        kb.check(lib, lib.kmb_scan1d_bwd(C.byref(eb)))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for _ in range(args.e2e_steps):
            kb.check(lib, lib.kmb_scan1d_fwd(C.byref(ef)))
            kb.check(lib, lib.kmb_scan1d_bwd(C.byref(eb)))
        torch.cuda.synchronize()
        te = (time.perf_counter() - t0) / args.e2e_steps
        te = kmb_dist.max_over_ranks(te, world, device="cuda")
        e2e_val = global_bytes / te / 1e9
        lib.kmb_set_sync(0)

    pk, pk_kind = peaks()
    # config 2 (channel-shared B/C, 16-byte rows, D a multiple of 32) runs the
    # sequence-split kernels (plus their fixer launches when L is split)
    # unless KMB_SCAN1D_SEGMENTS=0 selects the whole-sequence ones
    seg_on = os.environ.get("KMB_SCAN1D_SEGMENTS", "") != "0"
    n_seg, seg_len = C.c_int(1), C.c_int(0)
    kb.check(lib, lib.kmb_scan1d_seg_plan(BATCH, L, D, C.byref(n_seg), C.byref(seg_len)))
    fwd_name, bwd_name = (("k_scan1d_fwd_seg", "k_scan1d_bwd_seg") if seg_on
                          else ("k_scan1d_fwd", "k_scan1d_bwd_sh"))
    launches_per_step = 4 if seg_on and n_seg.value > 1 else 2
    dom_ms, dom_bytes, dom_name = ((bwd_ms, BWD_BYTES, bwd_name) if bwd_ms >= fwd_ms
                                   else (fwd_ms, FWD_BYTES, fwd_name))
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    tr = traffic_from_profile()
    traffic = None
    if tr and dom_name in tr:
        traffic = tr[dom_name]

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            nth = cpu_threads()
            secs, nch, kind = cpu_reference_run(nth, 1, 3, seed=100)
            cpu = {"value": bytes_for_channels(nch) / secs / 1e9, "unit": "GB/s", "cores": nth,
                   "kind": kind, "sample": cpu_sample_desc(nth) +
                   f", 3 timed passes of {secs:.2f} s"}
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": elapsed / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.shard_batch else "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (config-2 distributions, seeded per rank)",
            "config": {"workload": WORKLOAD, "batch_per_gpu": BATCH,
                       "global_batch": global_batch if args.shard_batch else BATCH * world,
                       "L": L, "D": D, "N": N,
                       "l_segments": n_seg.value if seg_on else 1,
                       "parallelism": (f"dp{world} ({'the config batch split over the ranks' if args.shard_batch else 'independent batch per rank'}; "
                                       "dA all-reduced by the library's NCCL communicator on a "
                                       "side stream, overlapped with the next forward)"),
                       "l2": "inputs larger than L2 (each [B,L,D] tensor is 201 MB)",
                       "fwd_ms": fwd_ms, "bwd_ms": bwd_ms,
                       "fwd_GBps": FWD_BYTES / fwd_ms / 1e6, "bwd_GBps": BWD_BYTES / bwd_ms / 1e6},
            "roofline": {"bound": "hbm", "kernel": dom_name, "achieved": achieved,
                         "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
                         "peak_source": f"{pk_kind} hbm_gbs (MEASURED_PEAKS.json)",
                         "algorithmic_bytes_per_launch": dom_bytes, "traffic": traffic},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_val, "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h,
                    "path": "kmb_scan1d_fwd + kmb_scan1d_bwd on pinned host buffers "
                            "(staged through the library's device pool)"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if ctx:
        lib.kmamba_distributed_fini_nccl(ctx)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
