"""Pins the CPU oracle (the checker of every GPU parity test) against the
reference: the known answers of the reference's own unit tests, its
finite-difference method, and golden outputs of the reference C sources
(tests/golden, made by make_golden.py from oracle/_ref)."""
import numpy as np
import pytest

from conftest import rel_err

f32 = np.float32
LN2, LN3 = np.log(f32(2)), np.log(f32(3))


# ---------------------------------------------------------------- known answers

def test_scannd_known_answer_2d(oracle):
    # tests/unit/test_scan_nd.c:41-90
    x = np.ones((4, 1), f32)
    A = np.array([LN2, LN3], f32).reshape(2, 1, 1)
    y, _ = oracle.scannd_fwd([2, 2], x, A, np.ones((4, 1, 1)), np.ones((4, 1, 1)),
                             np.ones((2, 4, 1)))
    np.testing.assert_allclose(y[:, 0], [1, 4, 3, 18], atol=1e-5)


def test_scan2d_known_answer(oracle):
    # the same case through the scan2d (asm) order, which scannd() dispatches to
    y, _ = oracle.scan2d_fwd(np.ones((4, 1)), np.full((1, 1), LN2), np.full((1, 1), LN3),
                             np.ones((4, 1, 1)), np.ones((4, 1, 1)), np.ones((4, 1)),
                             np.ones((4, 1)), 2, 2)
    np.testing.assert_allclose(y[:, 0], [1, 4, 3, 18], atol=1e-5)


def test_scannd_known_answer_3d(oracle):
    # tests/unit/test_scan_nd.c:92-140
    y, _ = oracle.scannd_fwd([2, 2, 2], np.ones((8, 1)), np.zeros((3, 1, 1)),
                             np.ones((8, 1, 1)), np.ones((8, 1, 1)), np.ones((3, 8, 1)))
    np.testing.assert_allclose(y[:, 0], [1, 2, 2, 5, 2, 5, 5, 16], atol=1e-5)


def test_convnd_known_answer_2d(oracle):
    # tests/unit/test_convnd_full.c:14-55
    out = oracle.convnd_fwd([2, 2], 2, np.array([[1], [2], [3], [4]], f32),
                            np.array([[1], [2], [3], [4]], f32), np.array([0.5], f32))
    np.testing.assert_allclose(out[:, 0], [4.5, 11.5, 14.5, 30.5], atol=1e-5)


def test_wavefront_known_answers(oracle):
    # tests/unit/test_wavefront_nd.c:104-150
    ls, _ = oracle.wavefront_plan([3, 4])
    assert list(np.diff(ls)) == [1, 2, 3, 3, 2, 1]
    ls, lo = oracle.wavefront_plan([2, 3, 2])
    assert list(np.diff(ls)) == [1, 3, 4, 3, 1]
    assert sorted(lo) == list(range(12))


def _scan1d_test_ref(x, A, B, Cm, dt):
    """The scalar C reference of tests/unit/test_scan1d.c:33-66 in float32."""
    L, D = x.shape
    M = A.shape[1]
    state = np.zeros((D, M), f32)
    y = np.zeros((L, D), f32)
    for t in range(L):
        dA = np.exp(dt[t][:, None] * A).astype(f32)
        bbar = (dt[t][:, None] * B[t]).astype(f32)
        state = (dA * state + bbar * x[t][:, None]).astype(f32)
        y[t] = (Cm[t] * state).sum(axis=1, dtype=f32)
    return y, state


@pytest.mark.parametrize("L,D,M", [(4, 8, 1), (16, 16, 1), (64, 32, 1), (32, 24, 1),
                                   (4, 8, 2), (16, 16, 2)])
def test_scan1d_matches_reference_test_formula(oracle, L, D, M):
    # tests/unit/test_scan1d.c:213-224: asm vs C reference within 1e-5
    rng = np.random.default_rng(42 + L * D * M)
    x = rng.uniform(-1, 1, (L, D)).astype(f32)
    A = rng.uniform(-1, -0.01, (D, M)).astype(f32)
    B = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
    Cm = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
    dt = rng.uniform(0.01, 0.5, (L, D)).astype(f32)
    y, h, _ = oracle.scan1d_fwd(x, dt, A, B, Cm)
    y_ref, h_ref = _scan1d_test_ref(x, A, B, Cm, dt)
    assert np.all(np.isfinite(y))
    assert np.max(np.abs(y - y_ref)) <= 1e-5
    assert np.max(np.abs(h - h_ref)) <= 1e-5


def test_scan1d_zero_input(oracle):
    # tests/unit/test_scan1d.c:168-193
    L, D, M = 4, 8, 1
    y, h, _ = oracle.scan1d_fwd(np.zeros((L, D)), np.full((L, D), 0.1), np.full((D, M), -0.5),
                                np.zeros((L, D, M)), np.ones((L, D, M)))
    assert np.abs(y).sum() + np.abs(h).sum() < 1e-12


def test_scan1d_clamp_and_nan(oracle):
    # cpu/scan1d.asm:136-140: min(h,1000) then max(h,-1000); NaN -> +1000
    x = np.array([[1e6], [-1e7], [np.nan]], f32)
    y, h, h_all = oracle.scan1d_fwd(x, np.ones((3, 1)), np.full((1, 1), -1.0),
                                    np.ones((3, 1, 1)), np.ones((3, 1, 1)), want_h_all=True)
    assert h_all[0, 0, 0] == 1000.0
    assert h_all[1, 0, 0] == -1000.0
    assert h_all[2, 0, 0] == 1000.0


# ------------------------------------------------------ finite differences

def _fd_grads(oracle, x, A, B, Cm, dt, eps=1e-3):
    def loss():
        y, _, _ = oracle.scan1d_fwd(x, dt, A, B, Cm, clamp=False)
        return float(np.sum(y, dtype=np.float64))
    out = {}
    for name, arr in (("x", x), ("A", A), ("B", B), ("C", Cm), ("dt", dt)):
        g = np.zeros(arr.shape)
        flat = arr.reshape(-1)
        for i in range(flat.size):
            o = flat[i]
            flat[i] = o + eps
            lp = loss()
            flat[i] = o - eps
            lm = loss()
            flat[i] = o
            g.reshape(-1)[i] = (lp - lm) / (2 * eps)
        out[name] = g
    return out


@pytest.mark.parametrize("L,D,M", [(4, 8, 1), (8, 16, 1), (4, 8, 2), (8, 16, 2)])
def test_scan1d_backward_finite_differences(oracle, L, D, M):
    # tests/unit/test_scan1d_backward.c:124-220: eps 1e-3, tol 1e-3, loss = sum(y)
    rng = np.random.default_rng(7 + L + D + M)
    x = rng.uniform(-1, 1, (L, D)).astype(f32)
    A = rng.uniform(-1, -0.01, (D, M)).astype(f32)
    B = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
    Cm = rng.uniform(-0.5, 0.5, (L, D, M)).astype(f32)
    dt = rng.uniform(0.01, 0.5, (L, D)).astype(f32)
    _, _, h_all = oracle.scan1d_fwd(x, dt, A, B, Cm, clamp=False, want_h_all=True)
    dx, ddt, dA, dB, dC = oracle.scan1d_bwd(x, dt, A, B, Cm, h_all, np.ones((L, D), f32))
    fd = _fd_grads(oracle, x, A, B, Cm, dt)
    for name, ana in (("x", dx), ("A", dA), ("B", dB), ("C", dC), ("dt", ddt)):
        assert np.max(np.abs(ana - fd[name])) <= 1e-3, name


@pytest.mark.parametrize("dims,D,M", [([3, 4], 2, 2), ([2, 3, 2], 2, 3), ([5], 3, 2),
                                      ([2, 2, 2, 2], 1, 2)])
@pytest.mark.parametrize("shared", [False, True])
def test_scannd_backward_finite_differences(oracle, dims, D, M, shared):
    # the 2D/ND backward has no reference: the adjoint is pinned this way
    rng = np.random.default_rng(sum(dims) * 31 + D + M)
    nd = len(dims)
    Pn = int(np.prod(dims))
    x = rng.uniform(-1, 1, (Pn, D)).astype(np.float32)
    A = rng.uniform(-1, -0.1, (nd, D, M)).astype(np.float32)
    bshape = (Pn, M) if shared else (Pn, D, M)
    B = rng.uniform(-0.5, 0.5, bshape).astype(np.float32)
    Cm = rng.uniform(-0.5, 0.5, bshape).astype(np.float32)
    delta = rng.uniform(0.05, 0.4, (nd, Pn, D)).astype(np.float32)
    w = rng.uniform(-1, 1, (Pn, D))
    _, h = oracle.scannd_fwd(dims, x, A, B, Cm, delta, shared=shared)
    grads = oracle.scannd_bwd(dims, x, A, B, Cm, delta, h, w.astype(np.float32), shared=shared)

    def loss():
        y, _ = oracle.scannd_fwd(dims, x, A, B, Cm, delta, shared=shared)
        return float(np.sum(y * w))
    eps = 1e-3
    for arr, ana in zip((x, A, B, Cm, delta), grads[:4] + (grads[4],)):
        fd = np.zeros(arr.shape)
        flat = arr.reshape(-1)
        for i in range(flat.size):
            o = flat[i]
            flat[i] = o + eps
            lp = loss()
            flat[i] = o - eps
            lm = loss()
            flat[i] = o
            fd.reshape(-1)[i] = (lp - lm) / (2 * eps)
        assert np.max(np.abs(ana - fd)) <= 2e-3


# ----------------------------------------------------- golden (reference C)

def test_scan1d_backward_matches_reference_bitwise(oracle, golden):
    for tag, c in golden("scan1d_bwd.npz").items():
        dx, ddt, dA, dB, dC = oracle.scan1d_bwd(c["x"], c["dt"], c["A"], c["B"], c["C"],
                                                c["h"], c["dy"], h0=c["h0"])
        for name, got in (("dx", dx), ("ddelta", ddt), ("dA", dA), ("dB", dB), ("dC", dC)):
            np.testing.assert_array_equal(got, c[name], err_msg=f"{tag} {name}")


def test_scannd_matches_reference_bitwise(oracle, golden):
    for tag, c in golden("scannd.npz").items():
        y, h = oracle.scannd_fwd(c["dims"], c["x"], c["A"], c["B"], c["C"], c["delta"])
        np.testing.assert_array_equal(y, c["y"], err_msg=tag)
        np.testing.assert_array_equal(h, c["h"], err_msg=tag)


def test_scan2d_order_matches_scannd_within_tolerance(oracle, golden):
    # scan2d (asm order) and scannd_ref associate differently; same math
    for tag, c in golden("scannd.npz").items():
        if len(c["dims"]) != 2:
            continue
        d1, d2 = map(int, c["dims"])
        y, h = oracle.scan2d_fwd(c["x"], c["A"][0], c["A"][1], c["B"], c["C"], c["delta"][0],
                                 c["delta"][1], d1, d2)
        assert rel_err(y, c["y"]) < 1e-5, tag


def test_convnd_matches_reference_bitwise(oracle, golden):
    for tag, c in golden("convnd.npz").items():
        K = int(tag.split("_K")[1])
        out = oracle.convnd_fwd(c["dims"], K, c["input"], c["kernel"], c["bias"])
        np.testing.assert_array_equal(out, c["output"], err_msg=tag)
        din, dk, db = oracle.convnd_bwd(c["dims"], K, c["input"], c["kernel"], c["dy"])
        np.testing.assert_array_equal(din, c["dinput"], err_msg=tag)
        np.testing.assert_array_equal(dk, c["dkernel"], err_msg=tag)
        np.testing.assert_array_equal(db, c["dbias"], err_msg=tag)


def test_plans_match_reference(oracle, golden):
    for tag, c in golden("plans.npz").items():
        ls, lo = oracle.wavefront_plan(c["dims"])
        np.testing.assert_array_equal(ls, c["level_starts"], err_msg=tag)
        np.testing.assert_array_equal(lo, c["level_offsets"], err_msg=tag)
