"""GPU parity of the ND / 2D selective scans with stored states (scannd,
scannd_ref*, om_scannd_forward, scan2d, kmb_scannd_*) against the
reference's golden outputs, its known answers and the CPU oracle."""
import ctypes as C

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL = 1e-4
LN2, LN3 = np.log(f32(2)), np.log(f32(3))
P_ = lambda a: None if a is None else a.ctypes.data  # noqa: E731


def nd_params(dims, D, M, x, A, B, Cm, delta, h, y):
    dims = np.ascontiguousarray(dims, dtype=np.int64)
    p = kb.ScanNDParams(P_(dims), len(dims), D, M, P_(x), P_(A), P_(B), P_(Cm), P_(delta),
                        P_(h), P_(y), None, None)
    return p, dims


def declare(lib):
    for n in ("scannd", "scannd_ref", "om_scannd_forward", "mamba_scannd_cuda_forward",
              "scannd_validate"):
        getattr(lib, n).argtypes = [C.POINTER(kb.ScanNDParams)]
        getattr(lib, n).restype = C.c_int
    lib.scannd_ref_with_plan.argtypes = [C.POINTER(kb.ScanNDParams), C.POINTER(kb.KMWavefrontPlan)]
    lib.scannd_ref_with_plan.restype = C.c_int
    lib.scan2d.argtypes = [C.POINTER(kb.Scan2DParams)]
    lib.mamba_scan2d_forward.argtypes = [C.POINTER(kb.Scan2DParams)]
    lib.kmb_scannd_fwd.argtypes = [C.POINTER(KmbScanND)]
    lib.kmb_scannd_bwd.argtypes = [C.POINTER(KmbScanND)]


class KmbScanND(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "delta", "A", "B", "C", "h", "y", "dy", "dx",
                                          "ddelta", "dA", "dB", "dC")] + [
        ("dims", C.c_long * 8), ("ndims", C.c_long), ("batch", C.c_long), ("D", C.c_long),
        ("M", C.c_long), ("bc_shared", C.c_int), ("flags", C.c_int)]


def test_known_answers(lib, cuda):
    declare(lib)
    # tests/unit/test_scan_nd.c:41-90 (2D) and :92-140 (3D)
    for dims, A, expected in (([2, 2], np.array([LN2, LN3], f32), [1, 4, 3, 18]),
                              ([2, 2, 2], np.zeros(3, f32), [1, 2, 2, 5, 2, 5, 5, 16])):
        P = int(np.prod(dims))
        x = np.ones(P, f32)
        B = np.ones(P, f32)
        Cm = np.ones(P, f32)
        delta = np.ones(len(dims) * P, f32)
        h = np.zeros(P, f32)
        y = np.zeros(P, f32)
        p, keep = nd_params(dims, 1, 1, x, A, B, Cm, delta, h, y)
        for fn in ("scannd_ref", "scannd"):
            y[:] = 0
            assert getattr(lib, fn)(C.byref(p)) == 0, kb.last_error(lib)
            np.testing.assert_allclose(y, expected, atol=1e-5)
    # the same 2D case through scan2d (cpu/scan2d.asm contract)
    one = np.ones(4, f32)
    h = np.zeros(4, f32)
    y = np.zeros(4, f32)
    a1 = np.array([LN2], f32)
    a3 = np.array([LN3], f32)
    p2 = kb.Scan2DParams(P_(one), P_(a1), P_(a3), P_(one), P_(one), P_(one), P_(one), P_(h),
                         P_(y), 2, 2, 1, 1)
    lib.scan2d(C.byref(p2))
    np.testing.assert_allclose(y, [1, 4, 3, 18], atol=1e-5)


def test_validate_and_unsupported(lib, cuda):
    declare(lib)
    one = np.ones(4, f32)
    p, keep = nd_params([2, 0], 1, 1, one, one, one, one, one, one, one)
    assert lib.scannd_validate(C.byref(p)) == 0
    assert lib.scannd(C.byref(p)) == -1
    p, keep = nd_params([2, 2], 1, 1, one, one, one, one, np.ones(8, f32), one.copy(), one.copy())
    assert lib.scannd_validate(C.byref(p)) == 1
    lam = np.ones(4, f32)
    p.lambda_ = lam.ctypes.data
    assert lib.scannd(C.byref(p)) == -1  # Mamba-3 branch not supported: loud -1


def test_golden_reference_scannd(lib, cuda, golden):
    declare(lib)
    for tag, c in golden("scannd.npz").items():
        P, D = c["x"].shape
        M = c["A"].shape[2]
        ins = {k: np.ascontiguousarray(c[k]) for k in ("x", "A", "B", "C", "delta")}
        h = np.full((P, D, M), np.nan, f32)
        y = np.full((P, D), np.nan, f32)
        p, keep = nd_params(c["dims"], D, M, ins["x"], ins["A"], ins["B"], ins["C"],
                            ins["delta"], h, y)
        assert lib.scannd(C.byref(p)) == 0, kb.last_error(lib)
        assert rel_err(y, c["y"]) <= TOL, tag
        assert rel_err(h, c["h"]) <= TOL, tag
        # with a prebuilt plan
        pl = lib.km_wavefront_plan_create(c["dims"].ctypes.data, len(c["dims"]))
        y2 = np.full((P, D), np.nan, f32)
        p.y = y2.ctypes.data
        assert lib.scannd_ref_with_plan(C.byref(p), pl) == 0
        lib.km_wavefront_plan_free(pl)
        assert rel_err(y2, c["y"]) <= TOL, tag


def test_om_scannd_device_pointers(lib, cuda, golden):
    import torch
    declare(lib)
    c = golden("scannd.npz")["3x4x5_D3_M2"]
    t = {k: torch.from_numpy(np.ascontiguousarray(c[k])).cuda() for k in ("x", "A", "B", "C",
                                                                          "delta")}
    h = torch.zeros(c["h"].shape, device="cuda")
    y = torch.zeros(c["y"].shape, device="cuda")
    dims = np.ascontiguousarray(c["dims"])
    p = kb.ScanNDParams(dims.ctypes.data, 3, 3, 2, t["x"].data_ptr(), t["A"].data_ptr(),
                        t["B"].data_ptr(), t["C"].data_ptr(), t["delta"].data_ptr(),
                        h.data_ptr(), y.data_ptr(), None, None)
    assert lib.om_scannd_forward(C.byref(p)) == 0
    assert lib.mamba_scannd_cuda_forward(C.byref(p)) == 0
    assert rel_err(y.cpu().numpy(), c["y"]) <= TOL


@pytest.mark.parametrize("d1,d2,D,M", [(5, 7, 3, 2), (16, 16, 8, 16), (1, 9, 2, 3), (33, 4, 5, 4)])
def test_scan2d_vs_oracle(lib, cuda, oracle, d1, d2, D, M):
    declare(lib)
    rng = np.random.default_rng(d1 * 100 + d2 + D + M)
    P = d1 * d2
    x = rng.normal(0, 1, (P, D)).astype(f32)
    A1 = (-np.exp(rng.uniform(0, np.log(16), (D, M)))).astype(f32)
    A2 = (-np.exp(rng.uniform(0, np.log(16), (D, M)))).astype(f32)
    B = rng.normal(0, 1, (P, D, M)).astype(f32)
    Cm = rng.normal(0, 1, (P, D, M)).astype(f32)
    dt = (np.log1p(np.exp(rng.normal(0, 1, (P, D)) - 2)) + np.log(2)).astype(f32)
    dt2 = (np.log1p(np.exp(rng.normal(0, 1, (P, D)) - 2)) + np.log(2)).astype(f32)
    y_ref, h_ref = oracle.scan2d_fwd(x, A1, A2, B, Cm, dt, dt2, d1, d2)
    h = np.full((P, D, M), np.nan, f32)
    y = np.full((P, D), np.nan, f32)
    p2 = kb.Scan2DParams(P_(x), P_(A1), P_(A2), P_(B), P_(Cm), P_(dt), P_(dt2), P_(h), P_(y),
                         d1, d2, D, M)
    lib.mamba_scan2d_forward(C.byref(p2))
    assert lib.kmb_last_status() == 0, kb.last_error(lib)
    assert rel_err(y, y_ref) <= TOL
    assert rel_err(h, h_ref) <= TOL


@pytest.mark.parametrize("dims,D,M,shared", [([6, 5], 4, 3, False), ([4, 4], 8, 16, True),
                                             ([3, 4, 5], 3, 2, True), ([2, 3, 2, 3], 2, 4, False),
                                             ([40], 5, 4, True), ([9, 13], 37, 5, True),
                                             # 2D wavefront kernels (channel-shared B/C,
                                             # M % 4 == 0 <= 16, D % 8 == 0): several
                                             # strips with a ragged last one, more rows
                                             # than the staging ring, M 8 and 12
                                             ([70, 130], 16, 16, True), ([9, 64], 8, 8, True),
                                             ([150, 20], 24, 12, True), ([1, 200], 8, 16, True),
                                             # warp-per-point 3D / 4D kernels (channel-shared
                                             # B/C, M % 4 == 0 <= 16, D % 8 == 0)
                                             ([5, 6, 7], 16, 16, True), ([4, 5, 3], 8, 4, True),
                                             ([9, 2, 10], 24, 12, True), ([8, 8, 8], 64, 16, True),
                                             ([3, 4, 5, 2], 8, 8, True), ([1, 7, 1], 8, 16, True),
                                             # staged gradient pass (M 16): axes of stride
                                             # > 64 fetched per stage (1, 2 and 3 such
                                             # axes, a stride just above 64), ranges of
                                             # 128 points with a ragged last one; M 8 on
                                             # the same grid takes the unstaged pass
                                             ([6, 9, 10], 8, 16, True), ([2, 5, 66], 16, 16, True),
                                             ([3, 70, 70], 8, 16, True), ([3, 3, 9, 10], 8, 16, True),
                                             ([2, 3, 5, 70], 8, 16, True),
                                             ([2, 3, 5, 70], 8, 8, True),
                                             # levels of up to ~1280 points: more than
                                             # one batch of 32 slots per warp in the
                                             # pipelined sweeps
                                             ([20, 64, 64], 8, 16, True)])
def test_batched_fwd_bwd_vs_oracle(lib, cuda, oracle, dims, D, M, shared, weak=False):
    import torch
    declare(lib)
    rng = np.random.default_rng(sum(dims) * 7 + D + M)
    batch, nd = 2, len(dims)
    P = int(np.prod(dims))
    x = rng.normal(0, 1, (batch, P, D)).astype(f32)
    A = (-np.exp(rng.uniform(0, np.log(16), (nd, D, M)))).astype(f32)
    bs = (batch, P, M) if shared else (batch, P, D, M)
    B = rng.normal(0, 1, bs).astype(f32)
    Cm = rng.normal(0, 1, bs).astype(f32)
    delta = (np.log1p(np.exp(rng.normal(0, 1, (batch, nd, P, D)) - 2)) + 0.3).astype(f32)
    if weak:
        # weak decays (|delta A log2 e| < 1/32, the polynomial path) in every
        # other point and on one channel everywhere; strong elsewhere
        delta[:, :, ::2, :] *= 1e-3
        delta[:, :, :, 1] = rng.uniform(1e-5, 1e-2, (batch, nd, P)).astype(f32)
    dy = rng.normal(0, 1, (batch, P, D)).astype(f32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    tx, tA, tB, tC, tdl, tdy = map(t, (x, A, B, Cm, delta, dy))
    th = torch.empty((batch, P, D, M), device="cuda")
    ty = torch.empty((batch, P, D), device="cuda")
    g = {k: torch.full(s, float("nan"), device="cuda") for k, s in
         (("dx", x.shape), ("ddelta", delta.shape), ("dA", A.shape), ("dB", B.shape),
          ("dC", B.shape))}
    a = KmbScanND()
    a.x, a.delta, a.A, a.B, a.C = (v.data_ptr() for v in (tx, tdl, tA, tB, tC))
    a.h, a.y, a.dy = th.data_ptr(), ty.data_ptr(), tdy.data_ptr()
    a.dx, a.ddelta, a.dA, a.dB, a.dC = (g[k].data_ptr() for k in ("dx", "ddelta", "dA", "dB", "dC"))
    for i, v in enumerate(dims):
        a.dims[i] = v
    a.ndims, a.batch, a.D, a.M, a.bc_shared = nd, batch, D, M, int(shared)
    kb.check(lib, lib.kmb_scannd_fwd(C.byref(a)))
    kb.check(lib, lib.kmb_scannd_bwd(C.byref(a)))
    dA_ref = np.zeros_like(A)
    for b in range(batch):
        y_ref, h_ref = oracle.scannd_fwd(dims, x[b], A, B[b], Cm[b], delta[b], shared=shared)
        assert rel_err(ty[b].cpu().numpy(), y_ref) <= TOL
        assert rel_err(th[b].cpu().numpy(), h_ref) <= TOL
        dx, dA, dB, dC, ddl = oracle.scannd_bwd(dims, x[b], A, B[b], Cm[b], delta[b], h_ref,
                                                dy[b], shared=shared)
        dA_ref += dA
        for name, want in (("dx", dx), ("dB", dB), ("dC", dC), ("ddelta", ddl)):
            assert rel_err(g[name][b].cpu().numpy(), want) <= TOL, name
    assert rel_err(g["dA"].cpu().numpy(), dA_ref) <= TOL


@pytest.mark.parametrize("dims,D,M", [([5, 6, 7], 16, 16), ([3, 4, 5, 2], 8, 8), ([6, 5], 8, 16),
                                      ([6, 9, 10], 8, 16), ([3, 4, 5, 2], 8, 16)])
def test_batched_weak_decays_vs_oracle(lib, cuda, oracle, dims, D, M):
    """The warp-per-point (3D / 4D) and 2D wavefront kernels with weak and
    strong decays mixed within a warp's points and channels: the
    warp-uniform MUFU-only shortcut must fall back to the weak-decay
    polynomial wherever a lane needs it."""
    test_batched_fwd_bwd_vs_oracle(lib, cuda, oracle, dims, D, M, True, weak=True)
