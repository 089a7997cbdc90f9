"""GPU parity at the BASELINE shapes that the smaller parametrised cases do
not reach, and of entry points the other files do not call directly:

- config 4 at its full shape (2D scan 256x256, batch 8, D 256, N 16, B/C
  shared, the same dt on both axes): every output of a 16-channel slice of
  every batch item, dA of that slice, and dB / dC (channel sums) of one
  whole item, against the CPU oracle;
- the config-5 volume (64^3, 3 axes) for the ND scan and the 3D ConvND at
  batch 1 with 64 channels, which runs the launch geometry of the
  1024-channel configuration (4096-point ranges in the staged gradient
  pass, full 64-channel conv tiles);
- om_convnd_forward / om_convnd_backward on device pointers;
- scan1d_backward_m1_shared_bc and its two asm-named aliases against the
  reference's own C implementation (oracle/_ref, cpu/scan1d_backward.c:
  23-191), with and without A_diag.

The oracle's C functions release the GIL (ctypes), so channel slices run
in a thread pool."""
import ctypes as C
from concurrent.futures import ThreadPoolExecutor
import os

import numpy as np
import pytest

from conftest import rel_err

import kmamba_b200 as kb

pytestmark = pytest.mark.gpu
f32 = np.float32
TOL = 1e-4


class KmbScanND(C.Structure):
    _fields_ = [(n, C.c_void_p) for n in ("x", "delta", "A", "B", "C", "h", "y", "dy", "dx",
                                          "ddelta", "dA", "dB", "dC")] + [
        ("dims", C.c_long * 8), ("ndims", C.c_long), ("batch", C.c_long), ("D", C.c_long),
        ("M", C.c_long), ("bc_shared", C.c_int), ("flags", C.c_int)]


def _pool():
    return ThreadPoolExecutor(max_workers=max(1, min(32, os.cpu_count() or 1)))


def _softplus(z):
    return np.log1p(np.exp(z))


def run_scannd(lib, dims, x, A, B, Cm, delta, dy):
    """kmb_scannd_fwd + kmb_scannd_bwd on device copies; returns the torch
    outputs (left on the device)."""
    import torch
    lib.kmb_scannd_fwd.argtypes = [C.POINTER(KmbScanND)]
    lib.kmb_scannd_bwd.argtypes = [C.POINTER(KmbScanND)]
    batch, P, D = x.shape
    nd, _, M = A.shape
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    tx, tA, tB, tC, tdl, tdy = map(t, (x, A, B, Cm, delta, dy))
    o = {"h": torch.empty((batch, P, D, M), device="cuda"),
         "y": torch.empty((batch, P, D), device="cuda")}
    for k, like in (("dx", tx), ("ddelta", tdl), ("dA", tA), ("dB", tB), ("dC", tC)):
        o[k] = torch.full_like(like, float("nan"))
    a = KmbScanND()
    a.x, a.delta, a.A, a.B, a.C = (v.data_ptr() for v in (tx, tdl, tA, tB, tC))
    a.h, a.y, a.dy = o["h"].data_ptr(), o["y"].data_ptr(), tdy.data_ptr()
    a.dx, a.ddelta, a.dA, a.dB, a.dC = (o[k].data_ptr() for k in ("dx", "ddelta", "dA", "dB",
                                                                   "dC"))
    for i, v in enumerate(dims):
        a.dims[i] = v
    a.ndims, a.batch, a.D, a.M, a.bc_shared = nd, batch, D, M, 1
    kb.check(lib, lib.kmb_scannd_fwd(C.byref(a)))
    kb.check(lib, lib.kmb_scannd_bwd(C.byref(a)))
    torch.cuda.synchronize()
    del tx, tA, tB, tC, tdl, tdy
    return o


def oracle_slice(oracle, dims, x, A, B, Cm, delta, dy, sl):
    """Oracle forward + adjoint of one batch item restricted to channels sl
    (B / C are shared across channels, so a slice is a complete problem)."""
    xs = np.ascontiguousarray(x[:, sl])
    As = np.ascontiguousarray(A[:, sl])
    ds = np.ascontiguousarray(delta[:, :, sl])
    ys = np.ascontiguousarray(dy[:, sl])
    y, h = oracle.scannd_fwd(dims, xs, As, B, Cm, ds, shared=True)
    dx, dA, dB, dC, ddl = oracle.scannd_bwd(dims, xs, As, B, Cm, ds, h, ys, shared=True)
    return dict(y=y, h=h, dx=dx, dA=dA, dB=dB, dC=dC, ddelta=ddl)


def nd_dA_f64(dims, x, A, B, Cm, delta, dy):
    """float64 dA of the ND recurrence (scannd semantics, channel-shared B/C)
    summed over the batch: the forward h and the adjoint g are swept level by
    level (every point of a wavefront level at once), then
    dA_a = sum_p g(p) delta_a(p) exp(delta_a(p) A_a) h(p - e_a).
    x, dy [nb, P, Ds]; A [nd, Ds, M]; B, C [nb, P, M]; delta [nb, nd, P, Ds]."""
    nd, P = len(dims), int(np.prod(dims))
    st = [int(np.prod(dims[a + 1:])) for a in range(nd)]
    co = np.indices(dims).reshape(nd, P)
    lvl = co.sum(0)
    order = np.argsort(lvl, kind="stable")
    bounds = np.searchsorted(lvl[order], np.arange(lvl.max() + 2))
    prev = [np.where(co[a] > 0, np.arange(P) - st[a], -1) for a in range(nd)]
    nxt = [np.where(co[a] < dims[a] - 1, np.arange(P) + st[a], -1) for a in range(nd)]
    f = np.float64
    xs = np.moveaxis(x.astype(f), 1, 0)                       # [P, nb, Ds]
    ys = np.moveaxis(dy.astype(f), 1, 0)
    dl = np.moveaxis(delta.astype(f), 2, 0)                   # [P, nb, nd, Ds]
    Bs, Cs = np.moveaxis(B.astype(f), 1, 0), np.moveaxis(Cm.astype(f), 1, 0)  # [P, nb, M]
    A64 = A.astype(f)
    dtbar = dl.sum(2) / nd
    h = np.zeros((P, x.shape[0], x.shape[2], A.shape[2]))
    for l in range(len(bounds) - 1):
        pts = order[bounds[l]:bounds[l + 1]]
        hn = (dtbar[pts] * xs[pts])[..., None] * Bs[pts][:, :, None, :]
        for a in range(nd):
            pp = prev[a][pts]
            ok = pp >= 0
            if ok.any():
                dec = np.exp(dl[pts[ok], :, a, :, None] * A64[a])
                hn[ok] += dec * h[pp[ok]]
        h[pts] = hn
    g = np.zeros_like(h)
    dA = np.zeros(A.shape)
    for l in range(len(bounds) - 2, -1, -1):
        pts = order[bounds[l]:bounds[l + 1]]
        gn = ys[pts][..., None] * Cs[pts][:, :, None, :]
        for a in range(nd):
            sp = nxt[a][pts]
            ok = sp >= 0
            if ok.any():
                gn[ok] += np.exp(dl[sp[ok], :, a, :, None] * A64[a]) * g[sp[ok]]
        g[pts] = gn
        for a in range(nd):
            pp = prev[a][pts]
            ok = pp >= 0
            if ok.any():
                da = dl[pts[ok], :, a, :, None]
                dA[a] += (gn[ok] * da * np.exp(da * A64[a]) * h[pp[ok]]).sum(axis=(0, 1))
    return dA


def test_config4_full_shape(lib, cuda, oracle):
    """256x256, batch 8, D 256, N 16, channel-shared
    B/C, dt = softplus(N(0,1) - 2) + ln 2 on both axes."""
    import torch
    dims, batch, D, M = [256, 256], 8, 256, 16
    P, nd = 256 * 256, 2
    rng = np.random.default_rng(4)
    x = rng.standard_normal((batch, P, D), dtype=f32)
    dt = (_softplus(rng.standard_normal((batch, 1, P, D), dtype=f32) - 2) + np.log(2)).astype(f32)
    delta = np.ascontiguousarray(np.concatenate([dt, dt], axis=1))
    del dt
    A = (-np.exp(rng.uniform(0, np.log(16), (nd, D, M)))).astype(f32)
    B = rng.standard_normal((batch, P, M), dtype=f32)
    Cm = rng.standard_normal((batch, P, M), dtype=f32)
    dy = rng.standard_normal((batch, P, D), dtype=f32)
    o = run_scannd(lib, dims, x, A, B, Cm, delta, dy)

    sl = slice(0, 16)        # checked on every batch item
    whole = 3                # every channel of this item (dB / dC channel sums)
    jobs = [(b, sl) for b in range(batch)] + [(whole, slice(c, c + 16))
                                              for c in range(16, D, 16)]
    with _pool() as ex:
        futs = {(b, s.start): ex.submit(oracle_slice, oracle, dims, x[b], A, B[b], Cm[b],
                                        delta[b], dy[b], s) for b, s in jobs}
        res = {k: f.result() for k, f in futs.items()}

    dA_ref = np.zeros((nd, 16, M), np.float64)
    for b in range(batch):
        r = res[(b, 0)]
        dA_ref += r["dA"]
        got = {"y": o["y"][b, :, sl], "h": o["h"][b, :, sl], "dx": o["dx"][b, :, sl],
               "ddelta": o["ddelta"][b, :, :, sl]}
        for k, v in got.items():
            assert rel_err(v.cpu().numpy(), r[k]) <= TOL, (b, k)
    # dA sums 8 x 65536 points per entry: held to the bar against a float64
    # sweep of the 16 checked channels, and to the fp32 oracle within that
    # oracle's own rounding of the long sums on the same channels
    dA64 = nd_dA_f64(dims, x[:, :, sl], A[:, sl], B, Cm, delta[:, :, :, sl], dy[:, :, sl])
    got_dA = o["dA"][:, sl].cpu().numpy()
    assert rel_err(got_dA, dA64) <= TOL
    assert rel_err(got_dA, dA_ref) <= TOL + rel_err(dA_ref, dA64)
    dB_ref = sum(res[(whole, c)]["dB"].astype(np.float64) for c in range(0, D, 16))
    dC_ref = sum(res[(whole, c)]["dC"].astype(np.float64) for c in range(0, D, 16))
    assert rel_err(o["dB"][whole].cpu().numpy(), dB_ref) <= TOL
    assert rel_err(o["dC"][whole].cpu().numpy(), dC_ref) <= TOL
    del o
    torch.cuda.empty_cache()


def test_nd3_64cube_scan_and_conv(lib, cuda, oracle):
    """The config-5 volume: 64^3 grid, 3 axes, batch 1, 64 channels, N 16
    (ND scan) and K 3 (ConvND), forward and backward, every output against
    the oracle."""
    import torch
    dims, D, M, K = [64, 64, 64], 64, 16, 3
    P, nd = 64 ** 3, 3
    rng = np.random.default_rng(5)
    x = rng.standard_normal((1, P, D), dtype=f32)
    delta = (_softplus(rng.standard_normal((1, nd, P, D), dtype=f32) - 2) +
             np.log(3)).astype(f32)
    A = (-np.exp(rng.uniform(0, np.log(16), (nd, D, M)))).astype(f32)
    B = rng.standard_normal((1, P, M), dtype=f32)
    Cm = rng.standard_normal((1, P, M), dtype=f32)
    dy = rng.standard_normal((1, P, D), dtype=f32)
    o = run_scannd(lib, dims, x, A, B, Cm, delta, dy)
    with _pool() as ex:
        futs = [ex.submit(oracle_slice, oracle, dims, x[0], A, B[0], Cm[0], delta[0], dy[0],
                          slice(c, c + 8)) for c in range(0, D, 8)]
        res = [f.result() for f in futs]
    for k, ax in (("y", 1), ("dx", 1), ("ddelta", 2)):
        want = np.concatenate([r[k] for r in res], axis=ax)
        assert rel_err(o[k][0].cpu().numpy(), want) <= TOL, k
    # dA sums 262144 points per entry, beyond what the fp32 oracle's own
    # sequential sums hold to 1e-4: every channel against a float64 sweep
    with _pool() as ex:
        parts = list(ex.map(lambda c: nd_dA_f64(dims, x[:, :, c:c + 8], A[:, c:c + 8], B, Cm,
                                                delta[:, :, :, c:c + 8], dy[:, :, c:c + 8]),
                            range(0, D, 8)))
    assert rel_err(o["dA"].cpu().numpy(), np.concatenate(parts, axis=1)) <= TOL
    for c, r in enumerate(res):
        assert rel_err(o["h"][0, :, 8 * c:8 * c + 8].cpu().numpy(), r["h"]) <= TOL, c
    dB_ref = sum(r["dB"].astype(np.float64) for r in res)
    dC_ref = sum(r["dC"].astype(np.float64) for r in res)
    assert rel_err(o["dB"][0].cpu().numpy(), dB_ref) <= TOL
    assert rel_err(o["dC"][0].cpu().numpy(), dC_ref) <= TOL
    del o
    torch.cuda.empty_cache()

    # 3D ConvND on the same volume
    ker = rng.normal(0, 1 / 5, (K ** 3, D)).astype(f32)
    bias = rng.normal(0, 0.1, (D,)).astype(f32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    ti, tk, tb, tdy = t(x), t(ker), t(bias), t(dy)
    out, din = torch.full_like(ti, float("nan")), torch.full_like(ti, float("nan"))
    dk, db = torch.full_like(tk, float("nan")), torch.full_like(tb, float("nan"))
    a = kb.KmbConvND()
    a.input, a.kernel, a.bias, a.output = (v.data_ptr() for v in (ti, tk, tb, out))
    a.dy, a.dinput, a.dkernel, a.dbias = (v.data_ptr() for v in (tdy, din, dk, db))
    for i, v in enumerate(dims):
        a.dims[i] = v
    a.ndims, a.batch, a.D, a.K = 3, 1, D, K
    kb.check(lib, lib.kmb_convnd_fwd(C.byref(a)))
    kb.check(lib, lib.kmb_convnd_bwd(C.byref(a)))
    torch.cuda.synchronize()

    def conv_slice(c):
        s = slice(c, c + 16)
        xi, ki = np.ascontiguousarray(x[0][:, s]), np.ascontiguousarray(ker[:, s])
        o_ = oracle.convnd_fwd(dims, K, xi, ki, bias[s])
        di, dki, dbi = oracle.convnd_bwd(dims, K, xi, ki, np.ascontiguousarray(dy[0][:, s]))
        return o_, di, dki, dbi

    with _pool() as ex:
        cres = list(ex.map(conv_slice, range(0, D, 16)))
    assert rel_err(out[0].cpu().numpy(), np.concatenate([r[0] for r in cres], 1)) <= TOL
    assert rel_err(din[0].cpu().numpy(), np.concatenate([r[1] for r in cres], 1)) <= TOL
    # dkernel / dbias sum over 262144 points: against float64 sums
    x4 = x[0].reshape(64, 64, 64, D).astype(np.float64)
    g4 = dy[0].reshape(64, 64, 64, D).astype(np.float64)
    dk64 = np.zeros((27, D))
    for k0 in range(3):
        for k1 in range(3):
            for k2 in range(3):
                s0, s1, s2 = 2 - k0, 2 - k1, 2 - k2
                dk64[(k0 * 3 + k1) * 3 + k2] = np.einsum(
                    "ijkd,ijkd->d", g4[s0:, s1:, s2:], x4[:64 - s0, :64 - s1, :64 - s2])
    assert rel_err(dk.cpu().numpy(), dk64) <= TOL
    assert rel_err(db.cpu().numpy(), g4.sum(axis=(0, 1, 2))) <= TOL
    dk_ref = np.concatenate([r[2] for r in cres], 1)
    assert rel_err(dk.cpu().numpy(), dk_ref) <= TOL + rel_err(dk_ref, dk64)


@pytest.mark.parametrize("dims,D,K", [([33, 17], 64, 3), ([9, 11], 5, 3), ([6, 5, 7], 8, 3),
                                      ([40], 16, 4)])
def test_om_convnd_device_pointers(lib, cuda, oracle, dims, D, K):
    """om_convnd_forward / om_convnd_backward (reference cuda/convnd.cu:258,
    332) with every tensor in device memory and dims on the host."""
    import torch
    rng = np.random.default_rng(sum(dims) + D + K)
    Pn = int(np.prod(dims))
    inp = rng.normal(0, 1, (Pn, D)).astype(f32)
    ker = rng.normal(0, 1 / 3, (K ** len(dims), D)).astype(f32)
    bias = rng.normal(0, 0.1, (D,)).astype(f32)
    dy = rng.normal(0, 1, (Pn, D)).astype(f32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    ti, tk, tb, tdy = t(inp), t(ker), t(bias), t(dy)
    out, din = torch.full_like(ti, float("nan")), torch.full_like(ti, float("nan"))
    dk, db = torch.full_like(tk, float("nan")), torch.full_like(tb, float("nan"))
    hd = np.ascontiguousarray(dims, dtype=np.int64)
    p = kb.ConvNDParams(ti.data_ptr(), tk.data_ptr(), tb.data_ptr(), out.data_ptr(),
                        tdy.data_ptr(), din.data_ptr(), dk.data_ptr(), db.data_ptr(),
                        hd.ctypes.data, len(dims), D, K)
    assert lib.om_convnd_forward(C.byref(p)) == 0, kb.last_error(lib)
    assert lib.om_convnd_backward(C.byref(p)) == 0, kb.last_error(lib)
    torch.cuda.synchronize()
    o = oracle.convnd_fwd(dims, K, inp, ker, bias)
    di, dki, dbi = oracle.convnd_bwd(dims, K, inp, ker, dy)
    assert rel_err(out.cpu().numpy(), o) <= TOL
    assert rel_err(din.cpu().numpy(), di) <= TOL
    assert rel_err(dk.cpu().numpy(), dki) <= 2 * TOL
    assert rel_err(db.cpu().numpy(), dbi) <= 2 * TOL
    # a NULL tensor is an error (-1), as in the reference
    p.dinput = None
    assert lib.om_convnd_backward(C.byref(p)) == -1


def _m1_problem(seed, L, D, with_diag):
    rng = np.random.default_rng(seed)
    x = rng.normal(0, 1, (L, D)).astype(f32)
    A = (-np.exp(rng.uniform(0, np.log(16), D))).astype(f32)
    B = rng.normal(0, 1, D).astype(f32)
    Cm = rng.normal(0, 1, D).astype(f32)
    delta = _softplus(rng.normal(0, 1, L) - 2).astype(f32)
    h0 = rng.normal(0, 1, D).astype(f32)
    dy = rng.normal(0, 1, (L, D)).astype(f32)
    # states of the forward the backward differentiates (float64, stored fp32)
    dA = np.exp(delta[:, None].astype(np.float64) * A[None, :].astype(np.float64))
    if with_diag:
        Ad = dA.astype(f32)
    else:
        Ad = None
    h = np.empty((L, D), f32)
    hp = h0.astype(np.float64)
    for t_ in range(L):
        hp = dA[t_] * hp + delta[t_] * B * x[t_]
        h[t_] = hp
    return dict(x=x, A=A, A_diag=Ad, B=B, C=Cm, delta=delta, h0=h0, h=h, dy=dy)


def _m1_params(q, outs):
    ptr = lambda a: None if a is None else a.ctypes.data  # noqa: E731
    L, D = q["x"].shape
    return kb.ScanBackwardSharedParams(
        ptr(q["x"]), ptr(q["A"]), ptr(q["A_diag"]), ptr(q["B"]), ptr(q["C"]), ptr(q["delta"]),
        ptr(q["h0"]), ptr(q["h"]), ptr(q["dy"]), ptr(outs["dx"]), ptr(outs["dA"]),
        ptr(outs["dB"]), ptr(outs["dC"]), ptr(outs["ddelta"]), L, D)


def _m1_outs(L, D):
    return {"dx": np.full((L, D), np.nan, f32), "dA": np.full(D, np.nan, f32),
            "dB": np.full(D, np.nan, f32), "dC": np.full(D, np.nan, f32),
            "ddelta": np.full(L, np.nan, f32)}


def _m1_f64(q):
    """float64 restatement of cpu/scan1d_backward.c:23-69."""
    L, D = q["x"].shape
    g = {k: np.asarray(v, np.float64) if v is not None else None for k, v in q.items()}
    dA_t = g["A_diag"] if g["A_diag"] is not None else np.exp(g["delta"][:, None] * g["A"])
    adj = np.zeros(D)
    out = {"dx": np.zeros((L, D)), "dA": np.zeros(D), "dB": np.zeros(D), "dC": np.zeros(D),
           "ddelta": np.zeros(L)}
    for t_ in range(L - 1, -1, -1):
        dt = g["delta"][t_]
        hp = g["h"][t_ - 1] if t_ > 0 else g["h0"]
        ah = adj + g["dy"][t_] * g["C"]
        out["dC"] += g["dy"][t_] * g["h"][t_]
        out["dB"] += ah * dt * g["x"][t_]
        out["dA"] += ah * dt * dA_t[t_] * hp
        out["dx"][t_] = ah * dt * g["B"]
        out["ddelta"][t_] = np.sum(ah * (g["A"] * dA_t[t_] * hp + g["B"] * g["x"][t_]))
        adj = ah * dA_t[t_]
    return out


@pytest.mark.parametrize("with_diag", [False, True])
@pytest.mark.parametrize("name", ["scan1d_backward_m1_shared_bc",
                                  "scan1d_backward_m1_shared_bc_asm",
                                  "scan1d_backward_m1_shared_bc_simple_asm"])
def test_m1_shared_bc_vs_reference(lib, cuda, oracle, name, with_diag):
    """Reference: cpu/scan1d_backward.c:23-191 compiled from the reference's
    own source (oracle/_ref).  The asm-named entry points (reference
    cpu/scan1d_backward_m1_shared_bc*.asm, which cannot be assembled here)
    compute the same gradients."""
    if not oracle.has_ref():
        pytest.skip("oracle/_ref (the reference's own C build) is not present")
    ref = oracle.ref_lib()
    kb.declare(ref)
    for seed, L, D in ((1, 300, 64), (2, 1000, 37)):
        q = _m1_problem(seed, L, D, with_diag)
        want = _m1_outs(L, D)
        ref.scan1d_backward_m1_shared_bc(C.byref(_m1_params(q, want)))
        got = _m1_outs(L, D)
        getattr(lib, name)(C.byref(_m1_params(q, got)))
        assert lib.kmb_last_status() == 0, kb.last_error(lib)
        want64 = _m1_f64(q)
        for k in want:
            # the reference's own fp32 sums (sequential in t, or over d) and
            # the GPU's agree with float64 to the bar; against each other the
            # bar adds the reference's own distance from float64
            assert rel_err(got[k], want64[k]) <= TOL, (k, rel_err(got[k], want64[k]))
            assert rel_err(got[k], want[k]) <= TOL + rel_err(want[k], want64[k]), k
