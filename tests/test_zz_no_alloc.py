"""kmb_scan1d_bwd_noalloc: the 1D scan backward for callers that cannot
allocate device memory during the call (their device memory belongs to
another allocator, or an allocation's implicit synchronisation is not
acceptable).  It keeps the forward checkpoints in the library's static
device scratch instead of a pooled buffer.

Checked through the C ABI against the allocating entry point
(kmb_scan1d_bwd with its internal checkpoint scratch), within the parity
tolerance of the other GPU tests, on two calls in a row with different
shapes, so the second call runs over the first one's leftover scratch.
This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL = 1e-4
NOALLOC_MAX = 2 * 1024 * 1024  # KMB_NOALLOC_CKPT_ELEMS


def problem(seed, bsz, L, D, N):
    import torch
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (bsz, L, D)).astype(f32)
    dt = np.log1p(np.exp(rng.normal(0, 1, (bsz, L, D)) - 2)).astype(f32)
    A = (-np.exp(rng.uniform(0, np.log(16), (D, N)))).astype(f32)
    B = rng.normal(0, 1, (bsz, L, N)).astype(f32)
    Cm = rng.normal(0, 1, (bsz, L, N)).astype(f32)
    dy = rng.normal(0, 1, (bsz, L, D)).astype(f32)
    t = {k: torch.from_numpy(v).cuda() for k, v in
         dict(x=x, dt=dt, A=A, B=B, C=Cm, dy=dy).items()}
    return t


def run(lib, t, fn):
    import torch
    bsz, L, D = t["x"].shape
    N = t["A"].shape[1]
    g = {k: torch.full(s, float("nan"), device="cuda") for k, s in
         (("dx", (bsz, L, D)), ("ddt", (bsz, L, D)), ("dA", (D, N)), ("dB", (bsz, L, N)),
          ("dC", (bsz, L, N)))}
    a = kb.KmbScan1D()
    a.x, a.dt, a.A, a.B, a.C, a.dy = (t[k].data_ptr() for k in ("x", "dt", "A", "B", "C", "dy"))
    a.dx, a.ddt, a.dA, a.dB, a.dC = (g[k].data_ptr() for k in ("dx", "ddt", "dA", "dB", "dC"))
    a.batch, a.L, a.D, a.N, a.bc_shared, a.clamp = bsz, L, D, N, 1, 1
    kb.check(lib, fn(C.byref(a)))
    torch.cuda.synchronize()
    return {k: v.cpu().numpy() for k, v in g.items()}


def test_noalloc_matches_allocating_backward_twice(lib, cuda):
    cases = [(11, 2, 300, 64, 16), (12, 1, 1000, 96, 16)]
    for seed, bsz, L, D, N in cases:
        assert lib.kmb_scan1d_ckpt_elems(bsz, L, D, N) <= NOALLOC_MAX
        t = problem(seed, bsz, L, D, N)
        want = run(lib, t, lib.kmb_scan1d_bwd)
        got = run(lib, t, lib.kmb_scan1d_bwd_noalloc)
        for k in want:
            assert np.all(np.isfinite(got[k])), k
            assert rel_err(got[k], want[k]) <= TOL, (seed, k)


def test_noalloc_rejects_oversized_and_host_buffers(lib, cuda):
    a = kb.KmbScan1D()
    # sizes beyond the static scratch: rejected before any pointer is used
    t = problem(13, 1, 64, 16, 16)
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
