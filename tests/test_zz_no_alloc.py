"""kmb_scan1d_bwd_noalloc: the 1D scan backward for callers that cannot
allocate device memory during the call (their device memory belongs to
another allocator, or an allocation's implicit synchronisation is not
acceptable).  It keeps the forward checkpoints in the library's static
device scratch instead of a pooled buffer.

Checked through the C ABI against the allocating entry point
(kmb_scan1d_bwd with its internal checkpoint scratch) and against the CPU
oracle (the reference's scan1d_backward restated), within the parity
tolerance of the other GPU tests.  Each check runs two calls in a row with
different shapes, so the second call runs over the first one's leftover
scratch; channel-shared and per-channel B/C and a non-zero initial state
are covered.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL = 1e-4
NOALLOC_MAX = 2 * 1024 * 1024  # KMB_NOALLOC_CKPT_ELEMS


def problem(seed, bsz, L, D, N, shared=True, with_h0=False):
    rng = np.random.default_rng(seed)
    bc = (bsz, L, N) if shared else (bsz, L, D, N)
    p = dict(x=rng.normal(0, 1, (bsz, L, D)).astype(f32),
             dt=np.log1p(np.exp(rng.normal(0, 1, (bsz, L, D)) - 2)).astype(f32),
             A=(-np.exp(rng.uniform(0, np.log(16), (D, N)))).astype(f32),
             B=rng.normal(0, 1, bc).astype(f32),
             C=rng.normal(0, 1, bc).astype(f32),
             dy=rng.normal(0, 1, (bsz, L, D)).astype(f32))
    if with_h0:
        p["h0"] = rng.normal(0, 1, (bsz, D, N)).astype(f32)
    p["shared"] = shared
    return p


def run(lib, p, fn):
    import torch
    t = {k: torch.from_numpy(v).cuda() for k, v in p.items() if isinstance(v, np.ndarray)}
    bsz, L, D = p["x"].shape
    N = p["A"].shape[1]
    g = {k: torch.full(s, float("nan"), device="cuda") for k, s in
         (("dx", (bsz, L, D)), ("ddt", (bsz, L, D)), ("dA", (D, N)), ("dB", p["B"].shape),
          ("dC", p["B"].shape))}
    a = kb.KmbScan1D()
    a.x, a.dt, a.A, a.B, a.C, a.dy = (t[k].data_ptr() for k in ("x", "dt", "A", "B", "C", "dy"))
    a.h0 = t["h0"].data_ptr() if "h0" in t else None
    a.dx, a.ddt, a.dA, a.dB, a.dC = (g[k].data_ptr() for k in ("dx", "ddt", "dA", "dB", "dC"))
    a.batch, a.L, a.D, a.N, a.clamp = bsz, L, D, N, 1
    a.bc_shared = 1 if p["shared"] else 0
    kb.check(lib, fn(C.byref(a)))
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in g.items()}


def oracle_grads(oracle, p):
    bsz = p["x"].shape[0]
    out = {"dx": [], "ddt": [], "dB": [], "dC": []}
    dA = np.zeros_like(p["A"], dtype=np.float64)
    for b in range(bsz):
        h0 = p["h0"][b] if "h0" in p else None
        _, _, h = oracle.scan1d_fwd(p["x"][b], p["dt"][b], p["A"], p["B"][b], p["C"][b],
                                    h0=h0, shared=p["shared"], want_h_all=True)
        dx, ddt, dAb, dB, dC = oracle.scan1d_bwd(p["x"][b], p["dt"][b], p["A"], p["B"][b],
                                                 p["C"][b], h, p["dy"][b], h0=h0,
                                                 shared=p["shared"])
        for k, v in (("dx", dx), ("ddt", ddt), ("dB", dB), ("dC", dC)):
            out[k].append(v)
        dA += dAb
    res = {k: np.stack(v) for k, v in out.items()}
    res["dA"] = dA
    return res


CASES = [  # seed, batch, L, D, N, channel-shared B/C, initial state h0
    (11, 2, 300, 64, 16, True, False),
    (12, 1, 1000, 96, 16, True, False),
    (14, 2, 203, 40, 16, False, True),
    (15, 1, 517, 24, 8, True, True),
]


def test_noalloc_matches_allocating_backward_twice(lib, cuda):
    for seed, bsz, L, D, N, shared, h0 in CASES:
        assert lib.kmb_scan1d_ckpt_elems(bsz, L, D, N) <= NOALLOC_MAX
        p = problem(seed, bsz, L, D, N, shared, h0)
        want = run(lib, p, lib.kmb_scan1d_bwd)
        got = run(lib, p, lib.kmb_scan1d_bwd_noalloc)
        for k in want:
            assert np.all(np.isfinite(got[k])), (seed, k)
            assert rel_err(got[k], want[k]) <= TOL, (seed, k)


def test_noalloc_matches_oracle(lib, cuda, oracle):
    for seed, bsz, L, D, N, shared, h0 in CASES[2:] + CASES[:1]:
        p = problem(seed, bsz, L, D, N, shared, h0)
        got = run(lib, p, lib.kmb_scan1d_bwd_noalloc)
        want = oracle_grads(oracle, p)
        for k in want:
            assert rel_err(got[k], want[k]) <= TOL, (seed, k, rel_err(got[k], want[k]))


def test_noalloc_rejects_oversized_and_host_buffers(lib, cuda):
    import torch
    a = kb.KmbScan1D()
    # sizes beyond the static scratch: rejected before any pointer is used
    t = {k: torch.from_numpy(v).cuda() for k, v in problem(13, 1, 64, 16, 16).items()
         if isinstance(v, np.ndarray)}
    a.x, a.dt, a.A, a.B, a.C, a.dy = (t[k].data_ptr() for k in ("x", "dt", "A", "B", "C", "dy"))
    a.dx = a.ddt = a.dA = a.dB = a.dC = t["x"].data_ptr()
    a.batch, a.L, a.D, a.N, a.bc_shared = 64, 4096, 1536, 16, 1
    assert lib.kmb_scan1d_bwd_noalloc(C.byref(a)) == kb.KMB_EUNSUPPORTED
    assert b"static scratch" in lib.kmb_last_error()
    # a host buffer would need a staging allocation: rejected
    host = np.zeros((1, 64, 16), f32)
    a.batch, a.L, a.D, a.N = 1, 64, 16, 16
    a.dy = host.ctypes.data
    assert lib.kmb_scan1d_bwd_noalloc(C.byref(a)) == kb.KMB_EINVAL
    assert b"device memory" in lib.kmb_last_error()
    # memory of another GPU is rejected too (needs two devices)
    if torch.cuda.device_count() > 1:
        other = torch.zeros((1, 64, 16), device="cuda:1")
        a.dy = other.data_ptr()
        assert lib.kmb_scan1d_bwd_noalloc(C.byref(a)) == kb.KMB_EINVAL
        assert b"current device" in lib.kmb_last_error()
